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
// bf16 path: the tcgen05 kernel of indexer_tk.cu.
//
// fp32 path: CUDA-core FFMA tiles (exact fp32 products, like the reference's
// fp32 einsum), used for fp32 modules.
#include "kernels.h"

namespace gsa {
namespace {

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
