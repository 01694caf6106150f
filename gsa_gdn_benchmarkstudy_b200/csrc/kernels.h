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

// ---- tcgen05 indexer with keys as the MMA's M dimension (indexer_tk.cu) and
// the fused indexer + top-k built on it.

// Per-row state of the fused selection.  The threshold kernel writes hi / lo
// and zeroes the counters; the kSelect pass adds to the counters.
struct SelectRowStats {
  float hi;    // keys scoring above hi are selected outright ("sure")
  float lo;    // keys scoring in [lo, hi] are candidates
  int sure;    // number of sure keys
  int ncand;   // candidates appended to the row's list
  int flags;   // kSelOverflow
  int pad[3];  // pad[0] of an indexer tile's first row: some row of the tile failed
};
static_assert(sizeof(SelectRowStats) == 32, "row stats are 32 bytes");
constexpr int kSelOverflow = 1;
constexpr int kSelCandCap = 2048;  // candidates of a row the fix-up can rank
constexpr int kSelMaxKeys = 65536;  // longest row of the fused selection (its bitmask in shared memory)

// A row of n causal keys needs the exact fallback when its candidates cannot
// hold the k-th key: more sure keys than k, fewer sure keys plus candidates
// than k, a candidate list that overflowed, or more candidates than the
// fix-up ranks.  Rows with n <= k select all their keys and never fail.
__host__ __device__ __forceinline__ bool select_row_failed(const SelectRowStats& st, int n,
                                                           int k) {
  if (n <= k) return false;
  return (st.flags & kSelOverflow) != 0 || st.sure > k || st.sure + st.ncand < k ||
         st.ncand > kSelCandCap;
}

enum IndexerTkMode { kIdxStore = 0, kIdxSample = 1, kIdxSelect = 2, kIdxStoreFailed = 3 };

struct IndexerTkArgs {
  const void* w;           // [B, Tq, 4] bf16, row stride w_stride
  int64_t w_stride;
  const float* bias;       // [4]
  float scale;
  int B, Tq, Tkv, q_pos0;
  int nkeys;               // keys of the launch (Tkv, or the number of sampled keys)
  int key_step, key_off;   // launch key i is sequence key i * key_step + key_off
  float* out;              // kStore / kSample / kStoreFailed: [B*Tq, out_stride] fp32
  int64_t out_stride;
  SelectRowStats* stats;   // kSelect / kStoreFailed: [B*Tq]
  // kSelect: the selection state of row r lives in the words
  // sel_bits[r*sel_stride, +sel_stride): its sure bits in [0, bitmask_words),
  // the candidate count of list l = 2 * (key chunk) + (chunk half) at
  // bitmask_words + l, and list l's cand_per_list entries (uint2 {score bits,
  // key}) from word cand_off + 2 * l * cand_per_list on.
  uint32_t* sel_bits;
  int64_t sel_stride;
  int64_t bitmask_words;
  int64_t cand_off;
  int cand_per_list;
  int k_sel;               // kStoreFailed: k of the failure test
  int* err;
};
// Tensor maps: q box {64, indexer_tk_rows_per_cta()}, k box {64, indexer_tk_keys_per_tile()};
// omap (kStore, kSample) is the fp32 score map {nkeys, Tq, B} with box {16, 32, 1} and
// 64-byte swizzle, unused by the other modes.
// A CTA covers indexer_tk_keys_per_cta() launch keys: two candidate lists.
int indexer_tk_rows_per_cta();
int indexer_tk_keys_per_tile();
int indexer_tk_keys_per_cta();
cudaError_t launch_indexer_tk(int mode, const CUtensorMap& qmap, const CUtensorMap& kmap,
                              const CUtensorMap& omap, const IndexerTkArgs& a,
                              cudaStream_t stream);

// Per row: from the row's sampled scores (samples[row * stride + i], i < the
// row's causal sample count, sample i = key i*key_step + key_off) estimate the
// k_sel-th score and write hi / lo thresholds around it (z standard
// deviations of the sample rank on each side) with zeroed counters.
cudaError_t launch_select_threshold(const float* samples, int64_t stride, int B, int Tq, int Tkv,
                                    int q_pos0, int key_step, int key_off, int k_sel, float z,
                                    SelectRowStats* stats, cudaStream_t stream);

// After the kSelect pass: marks, for kStoreFailed, each indexer tile of
// tile_rows rows that holds a failed row (in stats[first row of tile].pad[0]).
cudaError_t launch_select_scan(SelectRowStats* stats, int B, int Tq, int Tkv, int q_pos0,
                               int k_sel, int tile_rows, cudaStream_t stream);

// Per row: the exact top-k_sel from the sure bits and candidate lists of the
// kSelect pass (rank among candidates by (score desc, key asc)), or, for rows
// that failed, from their full score rows (written by kStoreFailed into the
// same workspace rows).  Outputs as launch_topk.  The lists are read with bulk
// copies: cand_off must be a multiple of 4 words and cand_per_list even.
cudaError_t launch_select_fixup(const uint32_t* ws, int64_t ws_stride, int64_t sel_words,
                                int64_t cand_off, int cand_per_list, int keys_per_chunk,
                                const SelectRowStats* stats, int B, int Tq, int Tkv, int q_pos0,
                                int k_sel, int32_t* indices, uint8_t* mask, uint32_t* bitmask,
                                int64_t bitmask_words, int* err, cudaStream_t stream);

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

// Fused projection GEMM (proj_gemm.cu): x [M, K] times the packed weight
// [n_tiles * 256, K] (both bf16, K-major), with RoPE on the q and k column
// tiles, the value gate on the v/vg tiles and the bias on the rest tiles.
struct ProjGemmArgs {
  int M;           // rows of x
  int K;           // reduction width (hidden size), a multiple of 64
  int n_tiles;     // 256-column tiles of the packed weight
  int q_tiles;     // tiles of q (and of k): hidden / 256
  int v_tiles;     // v/vg tiles: hidden / 128
  int rest_boxes;  // 64-column boxes of the rest output that hold columns
  int T;           // rows per sequence: row m has RoPE position pos0 + m % T
  int pos0;
  const __nv_bfloat16* cos;  // [*, 128] rotary tables
  const __nv_bfloat16* sin;
  const float* bias;         // [n_tiles * 256], packed like the weight
  int* err;
};
// Clusters of two CTAs that can be resident at once (0 on failure).
int proj_gemm_max_clusters();
// x / weight maps: 2-D, box {64, 128}; output maps: 2-D, box {64, 32}; all
// 128-byte swizzled.  `clusters` persistent clusters of two CTAs.
cudaError_t launch_proj_gemm(const CUtensorMap& xmap, const CUtensorMap& wmap,
                             const CUtensorMap& qmap, const CUtensorMap& kmap,
                             const CUtensorMap& vmap, const CUtensorMap& rmap,
                             const ProjGemmArgs& a, int clusters, cudaStream_t stream);

cudaError_t launch_gather_attention(const void* q, int64_t q_stride, const void* k,
                                    int64_t k_stride, const void* v, int64_t v_stride,
                                    const int32_t* indices, const uint8_t* mask, int k_sel,
                                    void* out, int64_t out_stride, float scale, int dtype, int B,
                                    int Tq, int Tkv, int H, int d, cudaStream_t stream);

}  // namespace gsa
