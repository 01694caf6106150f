// attn_gather.cu — index-gather sparse attention for explicit (indices, mask)
// inputs, fp32 online softmax.
//
// Reference: _gather_along_seq + sparse_attention_ref (gsa_ref.py:185-238)
// and the Triton _fused_sparse_attn_kernel (gsa_opt.py:199-346): for every
// (b, t, h), softmax over the selected slots of (q . K[idx] * scale), times
// V[idx]; indices clamped to [0, Tkv-1] (gsa_ref.py:196); masked slots take
// no part; a row whose slots are all masked yields zeros (nan_to_num at
// gsa_ref.py:235).  Unlike the Triton kernel, masked slots are skipped
// without loading their K/V rows, and duplicate indices count once per slot
// exactly as in the reference.
//
// One warp per (b, t, h): every lane owns d/32 consecutive channels.  A warp
// reads 32 (index, mask) pairs with one coalesced load, then works through
// the live slots eight at a time: the eight K and V row slices of a group are
// loaded together (sixteen independent vector loads per lane in flight, the
// rows mostly come from L2), the eight dot products are reduced across the
// warp together, and the online softmax takes the group in one step.  The
// kernel is bound by the L2/DRAM traffic of the gathered rows, 2 * d * sizeof
// per live slot and head.
#include "kernels.h"

namespace gsa {
namespace {

template <typename E, int D>
struct Lanes;

template <int D>
struct Lanes<__nv_bfloat16, D> {
  static constexpr int N = D / 32;  // channels per lane (2, 4 or 8)
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&x)[N]) {
    if constexpr (N == 8) {
      uint4 raw = *reinterpret_cast<const uint4*>(p);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = __bfloat162float(e[i]);
    } else if constexpr (N == 4) {
      uint2 raw = *reinterpret_cast<const uint2*>(p);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) x[i] = __bfloat162float(e[i]);
    } else {
      uint32_t raw = *reinterpret_cast<const uint32_t*>(p);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
      x[0] = __bfloat162float(e[0]);
      x[1] = __bfloat162float(e[1]);
    }
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, const float (&x)[N]) {
#pragma unroll
    for (int i = 0; i < N; i += 2)
      *reinterpret_cast<uint32_t*>(p + i) = pack_bf16x2(x[i], x[i + 1]);
  }
};

template <int D>
struct Lanes<float, D> {
  static constexpr int N = D / 32;
  static __device__ __forceinline__ void load(const float* p, float (&x)[N]) {
#pragma unroll
    for (int i = 0; i < N; i += 2) {
      const float2 v = *reinterpret_cast<const float2*>(p + i);
      x[i] = v.x;
      x[i + 1] = v.y;
    }
  }
  static __device__ __forceinline__ void store(float* p, const float (&x)[N]) {
#pragma unroll
    for (int i = 0; i < N; i += 2) *reinterpret_cast<float2*>(p + i) = make_float2(x[i], x[i + 1]);
  }
};

// A lane's N channels of one K or V row, kept as loaded (bf16 pairs or fp32)
// until they are used: half the registers of a float copy for bf16.
template <typename E, int N>
struct Raw {
  static constexpr int kWords = N * static_cast<int>(sizeof(E)) / 4;
  uint32_t w[kWords];
  __device__ __forceinline__ void load(const E* p) {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(p);
    if constexpr (kWords % 4 == 0) {
#pragma unroll
      for (int i = 0; i < kWords; i += 4) {
        const uint4 t = reinterpret_cast<const uint4*>(src)[i / 4];
        w[i] = t.x; w[i + 1] = t.y; w[i + 2] = t.z; w[i + 3] = t.w;
      }
    } else if constexpr (kWords == 2) {
      const uint2 t = *reinterpret_cast<const uint2*>(src);
      w[0] = t.x; w[1] = t.y;
    } else {
      w[0] = src[0];
    }
  }
  __device__ __forceinline__ float get(int e) const {
    if constexpr (sizeof(E) == 2) {
      const uint32_t x = w[e >> 1];
      return __uint_as_float((e & 1) ? (x & 0xFFFF0000u) : (x << 16));
    } else {
      return __uint_as_float(w[e]);
    }
  }
};

constexpr int kGroup = 8;  // live slots per step

template <typename E, int D>
__global__ void __launch_bounds__(256) gather_attn_kernel(
    const E* __restrict__ q, int64_t q_stride, const E* __restrict__ k, int64_t k_stride,
    const E* __restrict__ v, int64_t v_stride, const int32_t* __restrict__ indices,
    const uint8_t* __restrict__ mask, int k_sel, E* __restrict__ out, int64_t out_stride,
    float scale, int B, int Tq, int Tkv, int H) {
  using L = Lanes<E, D>;
  constexpr int N = L::N;
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= static_cast<int64_t>(B) * Tq * H) return;
  const int h = static_cast<int>(gw % H);
  const int64_t row = gw / H;  // b * Tq + t
  const int b = static_cast<int>(row / Tq);
  const int ch = h * D + lane * N;

  float qv[N];
  L::load(q + row * q_stride + ch, qv);
  float m = -INFINITY, l = 0.f, acc[N];
#pragma unroll
  for (int e = 0; e < N; ++e) acc[e] = 0.f;

  const int32_t* irow = indices + row * k_sel;
  const uint8_t* mrow = mask ? mask + row * k_sel : nullptr;
  const E* kb = k + static_cast<int64_t>(b) * Tkv * k_stride + ch;
  const E* vb = v + static_cast<int64_t>(b) * Tkv * v_stride + ch;

  for (int s0 = 0; s0 < k_sel; s0 += 32) {
    const int s = s0 + lane;
    int jl = 0;
    bool vl = false;
    if (s < k_sel) {
      jl = min(max(irow[s], 0), Tkv - 1);
      vl = mrow ? (mrow[s] != 0) : true;
    }
    uint32_t live = __ballot_sync(0xFFFFFFFFu, vl);
    while (live) {
      // the next (up to) kGroup live slots of this window
      int j[kGroup];
      int cnt = 0;
#pragma unroll
      for (int u = 0; u < kGroup; ++u) {
        const int src = live ? __ffs(live) - 1 : 0;
        j[u] = __shfl_sync(0xFFFFFFFFu, jl, src);
        cnt += live ? 1 : 0;
        live &= live - 1;
      }
      Raw<E, N> kv[kGroup], vv[kGroup];
#pragma unroll
      for (int u = 0; u < kGroup; ++u) {
        if (u < cnt) {
          kv[u].load(kb + static_cast<int64_t>(j[u]) * k_stride);
          vv[u].load(vb + static_cast<int64_t>(j[u]) * v_stride);
        }
      }
      float sc[kGroup];
#pragma unroll
      for (int u = 0; u < kGroup; ++u) {
        float part = 0.f;
        if (u < cnt) {
#pragma unroll
          for (int e = 0; e < N; ++e) part = fmaf(qv[e], kv[u].get(e), part);
        }
        sc[u] = part;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int u = 0; u < kGroup; ++u) sc[u] += __shfl_xor_sync(0xFFFFFFFFu, sc[u], o);
      }
      float gmax = -INFINITY;
#pragma unroll
      for (int u = 0; u < kGroup; ++u) {
        sc[u] = u < cnt ? sc[u] * scale : -INFINITY;
        gmax = fmaxf(gmax, sc[u]);
      }
      const float m_new = fmaxf(m, gmax);
      const float alpha = expf(m - m_new);  // 0 on the first live group (m = -inf)
      l *= alpha;
#pragma unroll
      for (int e = 0; e < N; ++e) acc[e] *= alpha;
#pragma unroll
      for (int u = 0; u < kGroup; ++u) {
        if (u < cnt) {
          const float p = expf(sc[u] - m_new);
          l += p;
#pragma unroll
          for (int e = 0; e < N; ++e) acc[e] = fmaf(p, vv[u].get(e), acc[e]);
        }
      }
      m = m_new;
    }
  }
  const float inv = l > 0.f ? 1.0f / l : 0.f;
#pragma unroll
  for (int e = 0; e < N; ++e) acc[e] *= inv;
  L::store(out + row * out_stride + ch, acc);
}

template <typename E>
cudaError_t launch_typed(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                         const void* v, int64_t v_stride, const int32_t* indices,
                         const uint8_t* mask, int k_sel, void* out, int64_t out_stride,
                         float scale, int B, int Tq, int Tkv, int H, int d, cudaStream_t stream) {
  const int64_t warps = static_cast<int64_t>(B) * Tq * H;
  const unsigned blocks = static_cast<unsigned>((warps * 32 + 255) / 256);
#define GSA_GATHER_CASE(DD)                                                                    \
  gather_attn_kernel<E, DD><<<blocks, 256, 0, stream>>>(                                       \
      static_cast<const E*>(q), q_stride, static_cast<const E*>(k), k_stride,                  \
      static_cast<const E*>(v), v_stride, indices, mask, k_sel, static_cast<E*>(out),          \
      out_stride, scale, B, Tq, Tkv, H)
  if (d == 64) GSA_GATHER_CASE(64);
  else if (d == 128) GSA_GATHER_CASE(128);
  else GSA_GATHER_CASE(256);
#undef GSA_GATHER_CASE
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gather_attention(const void* q, int64_t q_stride, const void* k,
                                    int64_t k_stride, const void* v, int64_t v_stride,
                                    const int32_t* indices, const uint8_t* mask, int k_sel,
                                    void* out, int64_t out_stride, float scale, int dtype, int B,
                                    int Tq, int Tkv, int H, int d, cudaStream_t stream) {
  if (B == 0 || Tq == 0 || H == 0) return cudaSuccess;
  if (dtype == GSA_DTYPE_BF16)
    return launch_typed<__nv_bfloat16>(q, q_stride, k, k_stride, v, v_stride, indices, mask,
                                       k_sel, out, out_stride, scale, B, Tq, Tkv, H, d, stream);
  return launch_typed<float>(q, q_stride, k, k_stride, v, v_stride, indices, mask, k_sel, out,
                             out_stride, scale, B, Tq, Tkv, H, d, stream);
}

}  // namespace gsa
