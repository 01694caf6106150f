// indexer.cu — gated lightning indexer scores.
//
//   out[b,r,j] = sum_h sigmoid(w[b,r,h]) * sigmoid(scale * q[b,r,h,:].k[b,j,:] + bias[h])
//   for j <= q_pos0 + r (causal), -inf above the diagonal.
//
// Reference: GatedLightningIndexer.forward, gsa_ref.py:97-126 (fp32 math on
// bf16-rounded projections; einsum, *scale, +bias, sigmoid, *sigmoid(w),
// sum over heads in order h = 0..3, masked_fill(-inf)).  The tensor-core
// epilogue uses sigmoid(z) = 1/2 + tanh(z/2)/2: with hw_h = sigmoid(w_h)/2,
// score = sum_h hw_h + sum_h hw_h * tanh(dot_h*scale/2 + bias_h/2), two keys
// per f32x2 FMA and one MUFU tanh.approx per key and head (the cheapest
// logistic on this SM: one MUFU op and two FMAs).  Scores come out about 1e-5
// (relative) from the reference's separately rounded fp32 ops, inside the
// 1e-2 bf16 budget.  The fp32 CUDA-core kernel keeps the reference's exact op
// order.
//
// bf16 path: tcgen05 tensor cores.  One CTA owns 128 query rows and a chunk
// of up to 512 keys.  Q (4 heads x [128 x 64] bf16) is loaded once by TMA
// with 128-byte swizzle; K sub-tiles of 32 keys stream through a 4-stage
// TMA ring.  Per sub-tile one thread issues 4 heads x 4 k-steps of
// tcgen05.mma (M=128, N=32, K=16) into one of two TMEM accumulator buffers
// (4 heads x 32 fp32 columns each; 256 columns per CTA so two CTAs share an
// SM).  Eight epilogue warps, two per TMEM lane quarter (thread = query row =
// TMEM lane), each read 16 of the 32 key columns of the four head
// accumulators with tcgen05.ld, apply the gated sum and the causal mask and
// store fp32 scores; at 94 registers, two 320-thread CTAs fit an SM.  Only
// key chunks at or below the diagonal run.
//
// fp32 path: CUDA-core FFMA tiles (exact fp32 products, like the reference's
// fp32 einsum), used for fp32 modules.
#include "kernels.h"

namespace gsa {
namespace {

constexpr int kIdxBM = 128;      // query rows per CTA
constexpr int kIdxBN = 32;       // keys per MMA sub-tile
constexpr int kIdxChunk = 512;   // keys per CTA
constexpr int kIdxStages = 4;    // K ring depth
constexpr int kIdxHeads = 4;
constexpr int kIdxD = 64;
constexpr int kIdxQBytes = kIdxBM * kIdxD * 2;    // 16 KB per head
constexpr int kIdxKBytes = kIdxBN * kIdxD * 2;    // 4 KB per stage
constexpr int kIdxTmemCols = 256;                 // 2 buffers x 4 heads x 32
constexpr int kIdxEpiWarps = 8;                   // two per TMEM lane quarter, 16 columns each
constexpr int kIdxTmaWarp = kIdxEpiWarps;         // warp 8: TMA producer
constexpr int kIdxMmaWarp = kIdxEpiWarps + 1;     // warp 9: MMA issuer, TMEM owner
constexpr int kIdxThreads = 32 * (kIdxEpiWarps + 2);
constexpr long long kIdxDrainCycles = 200000000LL;  // ~0.1 s after an abort

struct IdxSmem {
  uint64_t q_full;
  uint64_t k_full[kIdxStages];
  uint64_t k_empty[kIdxStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;  // MMAs in flight when the CTA gives up
  uint32_t tmem_base;
  int abort;
};
constexpr int kIdxSmemBytes =
    1024 /*align slack*/ + kIdxHeads * kIdxQBytes + kIdxStages * kIdxKBytes + 256;
static_assert(sizeof(IdxSmem) <= 256, "control block exceeds its 256-byte slot");

__global__ void __launch_bounds__(kIdxThreads, 2)
    indexer_tc_kernel(const __grid_constant__ CUtensorMap qmap,
                      const __grid_constant__ CUtensorMap kmap, IndexerArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* q_s = smem;                                   // 4 x 16 KB
  uint8_t* k_s = smem + kIdxHeads * kIdxQBytes;          // 4 x 4 KB
  IdxSmem* sh = reinterpret_cast<IdxSmem*>(k_s + kIdxStages * kIdxKBytes);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int n_qt = (a.Tq + kIdxBM - 1) / kIdxBM;
  const int qt = n_qt - 1 - static_cast<int>(blockIdx.y);  // heavy tiles first
  const int kc = blockIdx.x;
  const int b = blockIdx.z;
  const int row0 = qt * kIdxBM;
  const int maxpos = a.q_pos0 + min(row0 + kIdxBM - 1, a.Tq - 1);
  const int key_end = min(maxpos + 1, a.Tkv);           // exclusive
  const int key0 = kc * kIdxChunk;
  if (key0 >= key_end) return;  // chunk entirely above the diagonal
  const int nkeys = min(kIdxChunk, key_end - key0);
  const int nsub = (nkeys + kIdxBN - 1) / kIdxBN;

  if (tid == 0) {
    mbar_init(&sh->q_full, 1);
    for (int s = 0; s < kIdxStages; ++s) {
      mbar_init(&sh->k_full[s], 1);
      mbar_init(&sh->k_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sh->acc_full[s], 1);
      mbar_init(&sh->acc_empty[s], kIdxEpiWarps);
    }
    mbar_init(&sh->drain, 1);
    sh->abort = 0;
    fence_mbar_init();
  }
  if (warp == kIdxMmaWarp) {
    tmem_alloc(&sh->tmem_base, kIdxTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;
  volatile int* abort = &sh->abort;

  if (warp == kIdxTmaWarp) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&qmap);
      prefetch_tmap(&kmap);
      mbar_arrive_expect_tx(&sh->q_full, kIdxHeads * kIdxQBytes);
      for (int h = 0; h < kIdxHeads; ++h)
        tma_load_3d(q_s + h * kIdxQBytes, &qmap, h * kIdxD, row0, b, &sh->q_full);
      int s = 0;
      for (; s < nsub; ++s) {
        const int st = s % kIdxStages;
        const uint32_t ph = (s / kIdxStages) & 1;
        if (!mbar_wait(&sh->k_empty[st], ph ^ 1, a.err, abort)) break;
        mbar_arrive_expect_tx(&sh->k_full[st], kIdxKBytes);
        tma_load_3d(k_s + st * kIdxKBytes, &kmap, 0, key0 + s * kIdxBN, b, &sh->k_full[st]);
      }
      if (*abort) {  // let the copies this thread issued land before the CTA exits
        mbar_wait_drain(&sh->q_full, 0, kIdxDrainCycles);
        for (int ss = max(0, s - kIdxStages); ss < s; ++ss)
          mbar_wait_drain(&sh->k_full[ss % kIdxStages], (ss / kIdxStages) & 1, kIdxDrainCycles);
      }
    }
  } else if (warp == kIdxMmaWarp) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kIdxBM, kIdxBN, 0, 0);
      const uint32_t q_base = smem_u32(q_s);
      const uint32_t k_base = smem_u32(k_s);
      bool ok = mbar_wait(&sh->q_full, 0, a.err, abort);
      for (int s = 0; ok && s < nsub; ++s) {
        const int st = s % kIdxStages;
        const int buf = s & 1;
        if (!(ok = mbar_wait(&sh->k_full[st], (s / kIdxStages) & 1, a.err, abort))) break;
        if (!(ok = mbar_wait(&sh->acc_empty[buf], ((s >> 1) & 1) ^ 1, a.err, abort))) break;
        tc_fence_after();
#pragma unroll
        for (int h = 0; h < kIdxHeads; ++h) {
#pragma unroll
          for (int kk = 0; kk < kIdxD / 16; ++kk) {
            const uint64_t ad = sdesc_sw128(q_base + h * kIdxQBytes + kk * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(k_base + st * kIdxKBytes + kk * 32, 16, 1024);
            tc_mma_ss(tmem + buf * 128 + h * kIdxBN, ad, bd, idesc, kk > 0 ? 1u : 0u);
          }
        }
        tc_commit(&sh->k_empty[st]);
        tc_commit(&sh->acc_full[buf]);
      }
      if (!ok) {  // let the MMAs this thread issued finish before TMEM is freed
        tc_commit(&sh->drain);
        mbar_wait_drain(&sh->drain, 0, kIdxDrainCycles);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------ epilogue (warps 0-7)
    // Warp w reads TMEM lanes 32*(w%4).. (its query rows) and the 16 key
    // columns [16*(w/4), +16) of each 32-key sub-tile.
    const int i = (warp & 3) * 32 + lane;  // query row inside the tile == TMEM lane
    const int half = warp >> 2;
    const int r = row0 + i;
    const bool row_ok = r < a.Tq;
    const int pos = a.q_pos0 + r;
    // sigmoid(z) = 1/2 + tanh(z/2)/2, so with hw_h = sigmoid(w_h)/2:
    //   score = sum_h hw_h + sum_h hw_h * tanh(dot_h * scale/2 + bias_h/2)
    float hw[kIdxHeads], hb[kIdxHeads], hsum = 0.f;
#pragma unroll
    for (int h = 0; h < kIdxHeads; ++h) {
      float wv = 0.f;
      if (row_ok) {
        const __nv_bfloat16* wp = static_cast<const __nv_bfloat16*>(a.w) +
                                  (static_cast<int64_t>(b) * a.Tq + r) * a.w_stride + h;
        wv = __bfloat162float(*wp);
      }
      hw[h] = 0.5f * sigmoid_ref(wv);
      hb[h] = 0.5f * a.bias[h];
      hsum += hw[h];
    }
    const float hscale = 0.5f * a.scale;
    float* orow = a.out + (static_cast<int64_t>(b) * a.Tq + r) * a.out_stride;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    constexpr int kCols = kIdxBN / 2;
    for (int s = 0; s < nsub; ++s) {
      const int buf = s & 1;
      if (!mbar_wait_warp(&sh->acc_full[buf], (s >> 1) & 1, a.err, abort)) break;
      tc_fence_after();
      // two keys per f32x2 op; tanh on the MUFU
      uint64_t acc2[kCols / 2];
#pragma unroll
      for (int e = 0; e < kCols / 2; ++e) acc2[e] = f2_pack(hsum, hsum);
#pragma unroll
      for (int h = 0; h < kIdxHeads; ++h) {
        uint32_t raw[kCols];
        tmem_ld16(tmem + lane_base + buf * 128 + h * kIdxBN + half * kCols, raw);
        tc_wait_ld();
        const uint64_t zs = f2_pack(hscale, hscale);
        const uint64_t zb = f2_pack(hb[h], hb[h]);
        const uint64_t w2 = f2_pack(hw[h], hw[h]);
#pragma unroll
        for (int e = 0; e < kCols; e += 2) {
          const uint64_t z2 =
              f2_fma(f2_pack(__uint_as_float(raw[e]), __uint_as_float(raw[e + 1])), zs, zb);
          const uint64_t t2 = f2_pack(fast_tanh(f2_lo(z2)), fast_tanh(f2_hi(z2)));
          acc2[e >> 1] = f2_fma(t2, w2, acc2[e >> 1]);
        }
      }
      float acc[kCols];
#pragma unroll
      for (int e = 0; e < kCols; e += 2) {
        acc[e] = f2_lo(acc2[e >> 1]);
        acc[e + 1] = f2_hi(acc2[e >> 1]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->acc_empty[buf]);
      if (row_ok) {
        const int j0 = key0 + s * kIdxBN + half * kCols;
#pragma unroll
        for (int e = 0; e < kCols; ++e)
          if (j0 + e > pos) acc[e] = -INFINITY;
        if (j0 + kCols <= a.Tkv) {
          float4* dst = reinterpret_cast<float4*>(orow + j0);
#pragma unroll
          for (int v = 0; v < kCols / 4; ++v)
            dst[v] = make_float4(acc[4 * v], acc[4 * v + 1], acc[4 * v + 2], acc[4 * v + 3]);
        } else {
#pragma unroll
          for (int e = 0; e < kCols; ++e)
            if (j0 + e < a.Tkv) orow[j0 + e] = acc[e];
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kIdxMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kIdxTmemCols);
  }
}

// ---------------------------------------------------------------- fp32 / SIMT
constexpr int kSimtQ = 32;   // query rows per block
constexpr int kSimtK = 64;   // keys per block

template <typename E>
__global__ void __launch_bounds__(256) indexer_simt_kernel(
    const E* __restrict__ q, int64_t q_stride, const E* __restrict__ k, int64_t k_stride,
    const E* __restrict__ w, int64_t w_stride, const float* __restrict__ bias, float scale,
    int Tq, int Tkv, int q_pos0, int H_I, int d_I, float* __restrict__ out, int64_t out_stride) {
  extern __shared__ float fsm[];
  const int dp = d_I + 1;                    // padded row to avoid bank conflicts
  float* qs = fsm;                           // [kSimtQ][H_I][dp]
  float* ks = qs + kSimtQ * H_I * dp;        // [kSimtK][dp]
  float* sws = ks + kSimtK * dp;             // [kSimtQ][H_I]
  const int b = blockIdx.z;
  const int r0 = blockIdx.y * kSimtQ;
  const int j0 = blockIdx.x * kSimtK;
  const int maxpos = q_pos0 + min(r0 + kSimtQ - 1, Tq - 1);
  if (j0 > maxpos || j0 >= Tkv) return;
  const int tid = threadIdx.x;

  for (int idx = tid; idx < kSimtQ * H_I * d_I; idx += blockDim.x) {
    const int rr = idx / (H_I * d_I);
    const int rem = idx % (H_I * d_I);
    const int h = rem / d_I, e = rem % d_I;
    float v = 0.f;
    if (r0 + rr < Tq)
      v = static_cast<float>(q[(static_cast<int64_t>(b) * Tq + r0 + rr) * q_stride + h * d_I + e]);
    qs[(rr * H_I + h) * dp + e] = v;
  }
  for (int idx = tid; idx < kSimtK * d_I; idx += blockDim.x) {
    const int jj = idx / d_I, e = idx % d_I;
    float v = 0.f;
    if (j0 + jj < Tkv)
      v = static_cast<float>(k[(static_cast<int64_t>(b) * Tkv + j0 + jj) * k_stride + e]);
    ks[jj * dp + e] = v;
  }
  for (int idx = tid; idx < kSimtQ * H_I; idx += blockDim.x) {
    const int rr = idx / H_I, h = idx % H_I;
    float v = 0.f;
    if (r0 + rr < Tq) v = static_cast<float>(w[(static_cast<int64_t>(b) * Tq + r0 + rr) * w_stride + h]);
    sws[idx] = sigmoid_ref(v);
  }
  __syncthreads();

  // 256 threads: ty in [0,16) owns rows 2ty, 2ty+1; tx in [0,16) owns keys tx + 16c.
  const int ty = tid >> 4, tx = tid & 15;
#pragma unroll
  for (int ri = 0; ri < 2; ++ri) {
    const int rr = 2 * ty + ri;
    const int r = r0 + rr;
    if (r >= Tq) continue;
    const int pos = q_pos0 + r;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int jj = tx + 16 * c;
      const int j = j0 + jj;
      if (j >= Tkv) continue;
      float acc = 0.f;
      for (int h = 0; h < H_I; ++h) {
        const float* qv = qs + (rr * H_I + h) * dp;
        const float* kv = ks + jj * dp;
        float dot = 0.f;
        for (int e = 0; e < d_I; ++e) dot = fmaf(qv[e], kv[e], dot);
        const float z = __fadd_rn(__fmul_rn(dot, scale), bias[h]);
        const float g = __fmul_rn(sigmoid_ref(z), sws[rr * H_I + h]);
        acc = h == 0 ? g : __fadd_rn(acc, g);
      }
      out[(static_cast<int64_t>(b) * Tq + r) * out_stride + j] = j <= pos ? acc : -INFINITY;
    }
  }
}

__global__ void fill_upper_kernel(float* out, int64_t out_stride, int Tq, int Tkv, int q_pos0) {
  const int64_t row = blockIdx.x;  // b * Tq + r
  const int r = static_cast<int>(row % Tq);
  const int start = q_pos0 + r + 1;
  for (int j = start + threadIdx.x; j < Tkv; j += blockDim.x) out[row * out_stride + j] = -INFINITY;
}

}  // namespace

cudaError_t launch_indexer_tc(const CUtensorMap& qmap, const CUtensorMap& kmap,
                              const IndexerArgs& a, cudaStream_t stream) {
  if (a.B == 0 || a.Tq == 0 || a.Tkv == 0) return cudaSuccess;
  // once per device; two threads racing here both set the same attribute
  static std::atomic<bool> attr_set[kMaxDevices];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < kMaxDevices && !attr_set[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(indexer_tc_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kIdxSmemBytes);
    if (e != cudaSuccess) return e;
    attr_set[dev].store(true, std::memory_order_release);
  }
  const int n_qt = (a.Tq + kIdxBM - 1) / kIdxBM;
  const int max_key = min(a.q_pos0 + a.Tq, a.Tkv);
  const int n_kc = (max_key + kIdxChunk - 1) / kIdxChunk;
  dim3 grid(n_kc, n_qt, a.B);
  indexer_tc_kernel<<<grid, kIdxThreads, kIdxSmemBytes, stream>>>(qmap, kmap, a);
  return cudaGetLastError();
}

cudaError_t launch_indexer_simt(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                                const void* w, int64_t w_stride, const float* bias, float scale,
                                int dtype, int B, int Tq, int Tkv, int q_pos0, int H_I, int d_I,
                                float* out, int64_t out_stride, cudaStream_t stream) {
  if (B == 0 || Tq == 0 || Tkv == 0) return cudaSuccess;
  const int dp = d_I + 1;
  const size_t smem = sizeof(float) * (kSimtQ * H_I * dp + kSimtK * dp + kSimtQ * H_I);
  const int max_key = min(q_pos0 + Tq, Tkv);
  dim3 grid((max_key + kSimtK - 1) / kSimtK, (Tq + kSimtQ - 1) / kSimtQ, B);
  if (dtype == GSA_DTYPE_BF16) {
    auto kern = indexer_simt_kernel<__nv_bfloat16>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    kern<<<grid, 256, smem, stream>>>(
        static_cast<const __nv_bfloat16*>(q), q_stride, static_cast<const __nv_bfloat16*>(k),
        k_stride, static_cast<const __nv_bfloat16*>(w), w_stride, bias, scale, Tq, Tkv, q_pos0,
        H_I, d_I, out, out_stride);
  } else {
    auto kern = indexer_simt_kernel<float>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    kern<<<grid, 256, smem, stream>>>(static_cast<const float*>(q), q_stride,
                                      static_cast<const float*>(k), k_stride,
                                      static_cast<const float*>(w), w_stride, bias, scale, Tq, Tkv,
                                      q_pos0, H_I, d_I, out, out_stride);
  }
  return cudaGetLastError();
}

cudaError_t launch_fill_upper(float* out, int64_t out_stride, int B, int Tq, int Tkv, int q_pos0,
                              cudaStream_t stream) {
  if (B == 0 || Tq == 0 || Tkv == 0) return cudaSuccess;
  const int64_t rows = static_cast<int64_t>(B) * Tq;
  fill_upper_kernel<<<static_cast<unsigned>(rows), 256, 0, stream>>>(out, out_stride, Tq, Tkv,
                                                                     q_pos0);
  return cudaGetLastError();
}

}  // namespace gsa
