// rope_gates.cu — fused RoPE on q/k + ValueGate (G2) on v, and the
// element-wise OutputGate (G1).
//
// Reference semantics (bf16 module): every torch op rounds its result to
// bf16, so  q_embed = bf16( bf16(q*cos) + bf16(rotate_half(q)*sin) )
// (gsa_ref.py:29-40) and  v = bf16( v * bf16(sigmoid(vg)) )
// (gsa_ref.py:163-166).  The kernels below round at exactly those points;
// products of two bf16 values are exact in fp32, so the results match torch
// bit for bit except where sigmoid's float evaluation differs by an ulp.
// In the fp32 module every op rounds to fp32; __fmul_rn/__fadd_rn keep the
// compiler from contracting them into FMAs that torch does not perform.
#include "kernels.h"

namespace gsa {
namespace {

template <typename E>
struct Vec8;  // 8 elements, loaded/stored as 16- or 32-byte vectors

template <>
struct Vec8<__nv_bfloat16> {
  float v[8];
  __device__ __forceinline__ void load(const __nv_bfloat16* p) {
    uint4 raw = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(e[i]);
  }
  __device__ __forceinline__ void store(__nv_bfloat16* p) const {
    uint4 raw;
    uint32_t* w = reinterpret_cast<uint32_t*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = raw;
  }
  static __device__ __forceinline__ float round(float x) { return bf16_round(x); }
};

template <>
struct Vec8<float> {
  float v[8];
  __device__ __forceinline__ void load(const float* p) {
    float4 a = *reinterpret_cast<const float4*>(p);
    float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  __device__ __forceinline__ void store(float* p) const {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
  }
  static __device__ __forceinline__ float round(float x) { return x; }
};

// One thread = one (row, head, 8-wide chunk c of the first half); it also
// owns the matching chunk of the second half, the rotation partner.
template <typename E>
__global__ void __launch_bounds__(256) rope_gates_kernel(
    const E* __restrict__ q_src, const E* __restrict__ k_src, const E* __restrict__ v_src,
    const E* __restrict__ vg_src, int64_t src_stride, int B, int T, int H, int d,
    const E* __restrict__ cos_t, const E* __restrict__ sin_t, E* __restrict__ q_out,
    E* __restrict__ k_out, E* __restrict__ v_out) {
  using V = Vec8<E>;
  const int half = d >> 1;
  const int cph = half >> 3;  // chunks per half
  const int64_t total = static_cast<int64_t>(B) * T * H * cph;
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gid >= total) return;
  const int c = static_cast<int>(gid % cph);
  const int64_t rest = gid / cph;
  const int h = static_cast<int>(rest % H);
  const int64_t row = rest / H;
  const int t = static_cast<int>(row % T);

  const int64_t srow = row * src_stride;
  const int o1 = h * d + c * 8;
  const int o2 = o1 + half;
  const int64_t orow = row * static_cast<int64_t>(H) * d;

  V c1, c2, s1, s2;
  c1.load(cos_t + static_cast<int64_t>(t) * d + c * 8);
  c2.load(cos_t + static_cast<int64_t>(t) * d + half + c * 8);
  s1.load(sin_t + static_cast<int64_t>(t) * d + c * 8);
  s2.load(sin_t + static_cast<int64_t>(t) * d + half + c * 8);

  // q and k: x*cos + rotate_half(x)*sin, rotate_half(x) = cat(-x2, x1).
#pragma unroll
  for (int which = 0; which < 2; ++which) {
    const E* src = (which == 0 ? q_src : k_src) + srow;
    E* dst = which == 0 ? q_out : k_out;
    V x1, x2, y1, y2;
    x1.load(src + o1);
    x2.load(src + o2);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float a = V::round(__fmul_rn(x1.v[i], c1.v[i]));
      const float b = V::round(__fmul_rn(-x2.v[i], s1.v[i]));
      y1.v[i] = V::round(__fadd_rn(a, b));
      const float e = V::round(__fmul_rn(x2.v[i], c2.v[i]));
      const float f = V::round(__fmul_rn(x1.v[i], s2.v[i]));
      y2.v[i] = V::round(__fadd_rn(e, f));
    }
    y1.store(dst + orow + o1);
    y2.store(dst + orow + o2);
  }
  if (v_src == nullptr) return;

  // v * sigmoid(vg)
#pragma unroll
  for (int part = 0; part < 2; ++part) {
    const int o = part == 0 ? o1 : o2;
    V v, g, y;
    v.load(v_src + srow + o);
    g.load(vg_src + srow + o);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float gate = V::round(sigmoid_ref(g.v[i]));
      y.v[i] = V::round(__fmul_rn(v.v[i], gate));
    }
    y.store(v_out + orow + o);
  }
}

template <typename E>
__global__ void __launch_bounds__(256) output_gate_kernel(const E* __restrict__ o, int64_t o_stride,
                                                          const E* __restrict__ og,
                                                          int64_t og_stride, E* __restrict__ out,
                                                          int64_t out_stride, int rows, int width) {
  using V = Vec8<E>;
  const int cpr = width >> 3;
  const int64_t total = static_cast<int64_t>(rows) * cpr;
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gid >= total) return;
  const int c = static_cast<int>(gid % cpr);
  const int64_t r = gid / cpr;
  V a, g, y;
  a.load(o + r * o_stride + c * 8);
  g.load(og + r * og_stride + c * 8);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float gate = V::round(sigmoid_ref(g.v[i]));
    y.v[i] = V::round(__fmul_rn(a.v[i], gate));
  }
  y.store(out + r * out_stride + c * 8);
}

}  // namespace

cudaError_t launch_rope_gates(const void* q_src, const void* k_src, const void* v_src,
                              const void* vg_src, int64_t src_stride, int dtype, int B, int T,
                              int H, int d, const void* cos_t, const void* sin_t, void* q_out,
                              void* k_out, void* v_out, cudaStream_t stream) {
  const int64_t total = static_cast<int64_t>(B) * T * H * (d / 16);
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  const unsigned blocks = static_cast<unsigned>((total + threads - 1) / threads);
  if (dtype == GSA_DTYPE_BF16) {
    using E = __nv_bfloat16;
    rope_gates_kernel<E><<<blocks, threads, 0, stream>>>(
        static_cast<const E*>(q_src), static_cast<const E*>(k_src),
        static_cast<const E*>(v_src), static_cast<const E*>(vg_src), src_stride, B, T, H, d,
        static_cast<const E*>(cos_t), static_cast<const E*>(sin_t), static_cast<E*>(q_out),
        static_cast<E*>(k_out), static_cast<E*>(v_out));
  } else {
    using E = float;
    rope_gates_kernel<E><<<blocks, threads, 0, stream>>>(
        static_cast<const E*>(q_src), static_cast<const E*>(k_src),
        static_cast<const E*>(v_src), static_cast<const E*>(vg_src), src_stride, B, T, H, d,
        static_cast<const E*>(cos_t), static_cast<const E*>(sin_t), static_cast<E*>(q_out),
        static_cast<E*>(k_out), static_cast<E*>(v_out));
  }
  return cudaGetLastError();
}

cudaError_t launch_output_gate(const void* o, int64_t o_stride, const void* og, int64_t og_stride,
                               void* out, int64_t out_stride, int dtype, int rows, int width,
                               cudaStream_t stream) {
  const int64_t total = static_cast<int64_t>(rows) * (width / 8);
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  const unsigned blocks = static_cast<unsigned>((total + threads - 1) / threads);
  if (dtype == GSA_DTYPE_BF16) {
    using E = __nv_bfloat16;
    output_gate_kernel<E><<<blocks, threads, 0, stream>>>(
        static_cast<const E*>(o), o_stride, static_cast<const E*>(og), og_stride,
        static_cast<E*>(out), out_stride, rows, width);
  } else {
    output_gate_kernel<float><<<blocks, threads, 0, stream>>>(
        static_cast<const float*>(o), o_stride, static_cast<const float*>(og), og_stride,
        static_cast<float*>(out), out_stride, rows, width);
  }
  return cudaGetLastError();
}

}  // namespace gsa
