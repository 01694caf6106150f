// kernels.h — internal launchers behind the C ABI (include/gsa_b200.h).
// Argument checking happens in capi.cu; these assume valid arguments.
#pragma once

#include <atomic>

#include "common.cuh"

namespace gsa {

// Devices the per-device launch state covers (cudaGetDevice indices).
constexpr int kMaxDevices = 64;

cudaError_t launch_rope_gates(const void* q_src, const void* k_src, const void* v_src,
                              const void* vg_src, int64_t src_stride, int dtype, int B, int T,
                              int H, int d, const void* cos_t, const void* sin_t, void* q_out,
                              void* k_out, void* v_out, cudaStream_t stream);

cudaError_t launch_output_gate(const void* o, int64_t o_stride, const void* og, int64_t og_stride,
                               void* out, int64_t out_stride, int dtype, int rows, int width,
                               cudaStream_t stream);

// Tensor-core indexer (bf16, H_I = 4, d_I = 64).  Tensor maps are built by
// the caller (capi.cu).
struct IndexerArgs {
  const void* w;
  int64_t w_stride;
  const float* bias;
  float scale;
  int B, Tq, Tkv, q_pos0;
  float* out;
  int64_t out_stride;
  int* err;
};
cudaError_t launch_indexer_tc(const CUtensorMap& qmap, const CUtensorMap& kmap,
                              const IndexerArgs& a, cudaStream_t stream);

// CUDA-core indexer (fp32 or bf16 inputs, any H_I <= 8, d_I <= 128).
cudaError_t launch_indexer_simt(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                                const void* w, int64_t w_stride, const float* bias, float scale,
                                int dtype, int B, int Tq, int Tkv, int q_pos0, int H_I, int d_I,
                                float* out, int64_t out_stride, cudaStream_t stream);

// Writes -inf into out[b, r, j] for q_pos0 + r < j < Tkv.
cudaError_t launch_fill_upper(float* out, int64_t out_stride, int B, int Tq, int Tkv, int q_pos0,
                              cudaStream_t stream);

// Variance-based per-row k (adaptive mode).  k_row = clamp(floor(k_base *
// max(var_sum / var_rows, 1e-6) / max(row_var[row], 1e-6)), k_min, k_max).
// row_var == nullptr selects the fixed k of launch_topk's k_sel.
struct AdaptiveK {
  const float* row_var = nullptr;   // [B * Tq]
  const double* var_sum = nullptr;  // sum of row_var over all rows of the batch
  int64_t var_rows = 0;             // number of rows var_sum covers
  int k_base = 0, k_min = 0, k_max = 0;
  int32_t* row_k = nullptr;         // optional [B * Tq] output of k_row
};

// indices / mask rows are k_width slots wide (k_width >= the k of any row).
// finite_rows: the caller guarantees that no score in a row's valid columns
// is -inf (true for rows written by the indexer kernels).
cudaError_t launch_topk(const float* scores, int64_t score_stride, int B, int Tq, int Tkv,
                        int q_pos0, int k_sel, int k_width, const AdaptiveK& ad,
                        int32_t* indices, uint8_t* mask, uint32_t* bitmask,
                        int64_t bitmask_words, bool finite_rows, cudaStream_t stream);

// Per-row population variance of the finite scores among columns
// [0, min(q_pos0 + r + 1, Tkv)) into row_var[B * Tq], and their sum over all
// rows (summed in a fixed order, so repeat calls give the same bits) into
// *var_sum.
cudaError_t launch_row_variance(const float* scores, int64_t score_stride, int B, int Tq, int Tkv,
                                int q_pos0, float* row_var, double* var_sum, cudaStream_t stream);

struct MaskedAttnArgs {
  const uint32_t* bitmask;
  int64_t bitmask_words;
  const void* og;
  int64_t og_stride;
  void* out;
  int64_t out_stride;
  float scale;
  int B, Tq, Tkv, q_pos0, H;
  int* err;
};
// Registers per thread that the build gave masked_attn_kernel
// (cudaFuncGetAttributes), and in *expected the count its setmaxnreg split is
// written for.  launch_masked_attention refuses (cudaErrorNotSupported) to
// launch a build where the two differ: a split larger than the launch's
// allocation would wait for registers forever.
int masked_attention_regs(int* expected);
cudaError_t launch_masked_attention(const CUtensorMap& qmap, const CUtensorMap& kmap,
                                    const CUtensorMap& vmap, const MaskedAttnArgs& a,
                                    cudaStream_t stream);

cudaError_t launch_gather_attention(const void* q, int64_t q_stride, const void* k,
                                    int64_t k_stride, const void* v, int64_t v_stride,
                                    const int32_t* indices, const uint8_t* mask, int k_sel,
                                    void* out, int64_t out_stride, float scale, int dtype, int B,
                                    int Tq, int Tkv, int H, int d, cudaStream_t stream);

}  // namespace gsa
