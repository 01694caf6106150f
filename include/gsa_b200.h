/*
 * gsa_b200.h — C ABI of the B200 (sm_100a) Gated Sparse Attention forward.
 *
 * Every entry point takes raw device pointers, element strides, sizes and a
 * cudaStream_t passed as `void*` (NULL = legacy default stream).  Nothing in
 * this library allocates device memory: outputs and scratch buffers are
 * owned by the caller.  Every call returns a gsa_status_t; 0 means the work
 * was enqueued on `stream`.  Launch failures are reported as GSA_ERR_CUDA
 * and the CUDA error string is kept per host thread (gsa_last_error_string).
 *
 * Conventions shared by all entry points
 *   - B      batch size.
 *   - Tq     number of query rows handled by the call (a block of rows).
 *   - Tkv    number of key rows (the full causal key range).
 *   - q_pos0 absolute sequence position of query row 0 of the call; query
 *            row r has position q_pos0 + r and sees keys j <= q_pos0 + r.
 *            A whole-sequence call uses q_pos0 = 0 and Tq = Tkv.
 *   - *_stride arguments are in ELEMENTS between consecutive sequence rows
 *     of the same batch entry; batch entry b starts at b * T * stride.
 *   - dtype: GSA_DTYPE_BF16 or GSA_DTYPE_F32 (the module's parameter dtype).
 *
 * The reference interface each entry point replaces is cited as
 * file:line inside nirmalpratheep/GSA_GDN_BenchmarkStudy.
 */
#ifndef GSA_B200_H_
#define GSA_B200_H_

#include <stdint.h>
#include <stddef.h>

#if defined(__GNUC__)
#define GSA_API __attribute__((visibility("default")))
#else
#define GSA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  GSA_OK = 0,
  GSA_ERR_INVALID_ARG = 1,     /* null pointer, non-positive or inconsistent size */
  GSA_ERR_ALIGNMENT = 2,       /* pointer or stride breaks a 16-byte rule */
  GSA_ERR_UNSUPPORTED = 3,     /* shape/dtype this build does not implement */
  GSA_ERR_CUDA = 4,            /* a CUDA runtime/driver call failed */
  GSA_ERR_DEVICE_TIMEOUT = 5,  /* a bounded device-side wait expired */
  GSA_ERR_NO_DEVICE = 6        /* no usable sm_100 device */
} gsa_status_t;

typedef enum { GSA_DTYPE_BF16 = 0, GSA_DTYPE_F32 = 1 } gsa_dtype_t;

/* Library version, major*10000 + minor*100 + patch. */
GSA_API int gsa_version(void);

/* Human readable text for a status code (static storage). */
GSA_API const char* gsa_status_string(int status);

/* Text of the last CUDA error seen by a gsa_* call on this host thread. */
GSA_API const char* gsa_last_error_string(void);

/*
 * Reads (and optionally clears) the device-side error word that kernels set
 * when a bounded wait expires.  Synchronises the device.  *out receives 0 or
 * a GSA_ERR_* code.
 */
GSA_API int gsa_device_error(int* out, int reset);

/*
 * Fused RoPE (q and k) + ValueGate (G2).  Replaces gsa_ref.py:283-298 (q/k/v
 * views, ValueGate.forward at gsa_ref.py:163-166, apply_rotary_pos_emb at
 * gsa_ref.py:35-40) and the track_B block of gsa_opt.py:683-696.
 *
 *   q_src, k_src, v_src, vg_src  [B, T, H*d] (dtype), all with row stride
 *             src_stride; vg_src holds value-gate logits with the bias added.
 *             v_src and vg_src may both be NULL: then only RoPE runs.
 *   cos, sin  [T, d] (dtype) rotary tables; row t belongs to sequence row t
 *             of every batch entry.
 *   q_out, k_out, v_out  [B, T, H*d] contiguous (dtype).
 *
 *   q_out = dtype(dtype(q*cos) + dtype(rotate_half(q)*sin)), same for k,
 *   v_out = dtype(v * dtype(sigmoid(vg)))
 * Every product and sum is rounded to dtype where torch rounds it.
 * d must be a multiple of 16; rows and sources 16-byte aligned.
 */
GSA_API int gsa_rope_gates(const void* q_src, const void* k_src,
                           const void* v_src, const void* vg_src,
                           int64_t src_stride, int dtype,
                           int B, int T, int H, int d,
                           const void* cos, const void* sin,
                           void* q_out, void* k_out, void* v_out, void* stream);

/*
 * Gated lightning indexer scores.  Replaces GatedLightningIndexer.forward
 * score math (gsa_ref.py:104-124) and the Triton kernel wrapper
 * fused_gated_indexer (gsa_opt.py:143-176):
 *
 *   out[b,r,j] = sum_h sigmoid(w[b,r,h]) * sigmoid(q[b,r,h,:].k[b,j,:]*scale + bias[h])
 *
 * for j <= q_pos0 + r and j < Tkv; other columns are written only when
 * fill_upper != 0 (then with -inf, as the reference's masked_fill).
 *   q   [B, Tq, H_I, d_I] with row stride q_stride (dtype)
 *   k   [B, Tkv, d_I] with row stride k_stride (dtype)
 *   w   [B, Tq, H_I] with row stride w_stride (dtype; weight-proj bias added)
 *   bias [H_I] float32
 *   out [B, Tq, out_stride] float32, out_stride >= Tkv
 * bf16: tcgen05 tensor-core kernel, requires H_I == 4, d_I == 64, 16-byte
 * aligned rows.  f32: CUDA-core FFMA kernel (exact fp32 products).
 */
GSA_API int gsa_indexer_scores(const void* q, int64_t q_stride,
                       const void* k, int64_t k_stride,
                       const void* w, int64_t w_stride,
                       const float* bias, float scale, int dtype,
                       int B, int Tq, int Tkv, int q_pos0, int H_I, int d_I,
                       float* out, int64_t out_stride, int fill_upper,
                       void* stream);

/*
 * Top-k selector over causal indexer scores.  Replaces
 * AdaptiveTopKSelector.forward (gsa_ref.py:138-150, gsa_opt.py:473-483) and
 * the index sort of gsa_opt.py:674-677.
 *
 * Row r has n = min(q_pos0 + r + 1, Tkv) valid scores (columns 0..n-1).
 * If n <= k_sel all valid columns are selected, otherwise the k_sel largest,
 * ties (equal scores; -0.0 equals +0.0) broken toward the lower column
 * index.  Outputs (each may be NULL):
 *   indices [B, Tq, k_sel] int32: selected columns in ascending order, then
 *           (k_sel - selected) filler slots holding future positions
 *           min(n + s, Tkv - 1) with mask 0 (the reference's -inf slots)
 *   mask    [B, Tq, k_sel] uint8: 1 for selected slots
 *   bitmask [B, Tq, bitmask_words] uint32: bit j set iff column j selected;
 *           bitmask_words >= 4 * ceil(Tkv / 128), unused words written 0.
 * scores: [B, Tq, score_stride] float32.
 */
GSA_API int gsa_topk_select(const float* scores, int64_t score_stride,
                    int B, int Tq, int Tkv, int q_pos0, int k_sel,
                    int32_t* indices, uint8_t* mask,
                    uint32_t* bitmask, int64_t bitmask_words, void* stream);

/*
 * Adaptive k (opt-in; the reference module's selector always uses the fixed
 * k above).  The rule is the variance-based one of the reference's tutorial
 * notebook, gsa_explained.ipynb:575-592 ("Adaptive Top-K: How It Works"):
 *   var_r   = population variance of row r's valid scores (!= -inf) among
 *             columns [0, min(q_pos0 + r + 1, Tkv))
 *   avg_var = max(sum_r var_r / var_rows, 1e-6)    (mean over the batch)
 *   k_r     = clamp(floor(k_base * avg_var / max(var_r, 1e-6)), k_min, k_max)
 * and row r then selects its k_r largest scores as gsa_topk_select does.
 *
 * gsa_row_variance writes var_r to row_var [B*Tq] and the sum over the call's
 * rows to *var_sum (one double, 8-byte aligned; summed in a fixed order, so
 * the same inputs give the same bits).  A caller whose batch spans several
 * calls (row blocks, or ranks of a process group) adds their var_sum values
 * before selecting, and passes the total row count as var_rows.
 */
GSA_API int gsa_row_variance(const float* scores, int64_t score_stride,
                             int B, int Tq, int Tkv, int q_pos0,
                             float* row_var, double* var_sum, void* stream);

/* Slots per row of the index / mask outputs in adaptive mode:
 * min(k_max, Tkv).  No row selects more. */
GSA_API int gsa_adaptive_k_width(int k_max, int Tkv);

/*
 * Top-k selection with the per-row k_r above (replaces
 * AdaptiveTopKSelector.forward, gsa_ref.py:138-150, in adaptive mode).
 * Outputs as gsa_topk_select with rows gsa_adaptive_k_width(k_max, Tkv) slots
 * wide: the selected columns ascending, then masked filler.  row_k
 * [B*Tq] int32 (may be NULL) receives k_r.  Needs k_base >= 0,
 * 0 <= k_min <= k_max, k_max >= 1, var_rows >= 1.  A row whose k_r is 0
 * selects nothing.
 */
GSA_API int gsa_topk_select_adaptive(const float* scores, int64_t score_stride,
                                     int B, int Tq, int Tkv, int q_pos0,
                                     int k_base, int k_min, int k_max,
                                     const float* row_var, const double* var_sum,
                                     int64_t var_rows, int32_t* row_k,
                                     int32_t* indices, uint8_t* mask,
                                     uint32_t* bitmask, int64_t bitmask_words,
                                     void* stream);

/* Bytes of scratch gsa_indexer_topk_adaptive needs: the score rows of
 * gsa_indexer_topk_workspace_size plus the row variances and their sum. */
GSA_API int64_t gsa_indexer_topk_adaptive_workspace_size(int B, int Tq, int Tkv);

/*
 * gsa_indexer_topk in adaptive mode: indexer scores, gsa_row_variance over
 * the call's B*Tq rows (var_rows = B*Tq), gsa_topk_select_adaptive.  The
 * workspace (16-byte aligned) holds the scores, row variances and their sum.
 */
GSA_API int gsa_indexer_topk_adaptive(const void* q, int64_t q_stride,
                                      const void* k, int64_t k_stride,
                                      const void* w, int64_t w_stride,
                                      const float* bias, float scale, int dtype,
                                      int B, int Tq, int Tkv, int q_pos0, int H_I, int d_I,
                                      int k_base, int k_min, int k_max,
                                      void* workspace, int64_t workspace_bytes,
                                      int32_t* row_k, int32_t* indices, uint8_t* mask,
                                      uint32_t* bitmask, int64_t bitmask_words,
                                      void* stream);

/* Number of uint32 words per row that gsa_topk_select / gsa_masked_attention
 * expect for a key range of Tkv. */
GSA_API int64_t gsa_bitmask_words(int Tkv);

/* Bytes of caller-owned scratch that gsa_indexer_topk needs: B * Tq rows of
 * round-up-to-4(Tkv) floats (score rows, or a row's selection state) plus 32
 * bytes of per-row counters. */
GSA_API int64_t gsa_indexer_topk_workspace_size(int B, int Tq, int Tkv);

/*
 * Indexer scores followed by top-k selection in one call: the forward's
 * GatedLightningIndexer.forward (gsa_ref.py:97-126) + AdaptiveTopKSelector
 * (gsa_ref.py:138-150), the pair the reference runs back to back at
 * gsa_ref.py:303-308 / gsa_opt.py:664-677.  Arguments as for
 * gsa_indexer_scores and gsa_topk_select (any of indices / mask / bitmask
 * may be NULL); `workspace` holds workspace_bytes >=
 * gsa_indexer_topk_workspace_size bytes of caller-owned scratch.
 *
 * The selection equals gsa_topk_select applied to gsa_indexer_scores' output,
 * bit for bit.  With the fused selection (tensor-core path: bf16, H_I = 4,
 * d_I = 64; see gsa_set_fused_selection) the score matrix is never written:
 * each row's k-th score is bracketed from the row's scores against every 8th
 * key, one pass over all keys sets the bits of the keys above the bracket and
 * lists the few inside it, and a last pass ranks those exactly.  Rows whose
 * bracket misses are recomputed in full and selected from their scores, so
 * the result does not depend on the bracket.  Otherwise the causal score rows
 * are written to the workspace and selected from there.
 */
GSA_API int gsa_indexer_topk(const void* q, int64_t q_stride,
                             const void* k, int64_t k_stride,
                             const void* w, int64_t w_stride,
                             const float* bias, float scale, int dtype,
                             int B, int Tq, int Tkv, int q_pos0, int H_I, int d_I,
                             int k_sel, void* workspace, int64_t workspace_bytes,
                             int32_t* indices, uint8_t* mask,
                             uint32_t* bitmask, int64_t bitmask_words, void* stream);

/*
 * Which selection gsa_indexer_topk (and gsa_indexer_topk_noalloc) uses on the
 * tensor-core path, process-wide (no counterpart in the reference; a tuning
 * and testing knob).  Both give the same bits.
 *   GSA_FUSED_AUTO    the fused selection where it measured faster
 *                     (Tkv >= 16 * k_sel), scores + top-k elsewhere (default)
 *   GSA_FUSED_ALWAYS  the fused selection wherever it applies (Tkv > 2 * k_sel,
 *                     Tkv <= 65536)
 *   GSA_FUSED_NEVER   always scores + top-k
 * Returns GSA_ERR_INVALID_ARG for another mode.
 */
typedef enum { GSA_FUSED_AUTO = 0, GSA_FUSED_ALWAYS = 1, GSA_FUSED_NEVER = 2 } gsa_fused_mode_t;
GSA_API int gsa_set_fused_selection(int mode);

/* Size of the library's built-in scratch buffer for gsa_indexer_topk_noalloc:
 * gsa_indexer_topk_workspace_size(1, 2048, 2048), 16 MiB + 64 KiB. */
#define GSA_NOALLOC_SCRATCH_BYTES ((16ll << 20) + (64ll << 10))

/*
 * gsa_indexer_topk for callers that cannot allocate device memory.
 * This entry point has no counterpart in the reference.
 *
 * Some callers may not call cudaMalloc. Examples: a plugin inside a host
 * engine that owns every byte of device memory, or a runtime that fixes its
 * memory budget at start-up, since an allocation can synchronise the device
 * and fragment the pool. Such callers cannot provide the scratch that
 * gsa_indexer_topk takes as `workspace`. This variant keeps that scratch
 * instead in a buffer compiled into the library: GSA_NOALLOC_SCRATCH_BYTES
 * (16 MiB + 64 KiB) on every GPU that loads the library, held until the
 * process exits.
 * The caller still passes all inputs and outputs. Arguments are those of
 * gsa_indexer_topk without workspace / workspace_bytes.
 *
 *   - Size limit: the call needs gsa_indexer_topk_workspace_size(B, Tq, Tkv)
 *     bytes (B * Tq rows of round-up-to-4(Tkv) floats plus 32 bytes each; up
 *     to one 2048-token sequence).  Larger calls return GSA_ERR_UNSUPPORTED
 *     and say so in gsa_last_error_string(); use gsa_indexer_topk with a
 *     workspace then.
 *   - First call on a device: the first call of any gsa_* entry point on a
 *     device (this one included) looks up the device address of the buffer,
 *     once per device, with that device current.  Make that first call before
 *     any stream capture.  A device other than sm_100 gets GSA_ERR_NO_DEVICE.
 *   - Shared state: every call on a device uses the same buffer, which keeps
 *     the scratch of the last call.  Nothing in it needs to start at zero,
 *     because each call writes every score, bit and counter it reads.  Calls whose work
 *     overlaps on the GPU (e.g. on two streams) race on the buffer; order
 *     them on one stream or use gsa_indexer_topk.
 *   - Allocation: no cudaMalloc, cudaFree or allocating library routine is
 *     called.
 */
GSA_API int gsa_indexer_topk_noalloc(const void* q, int64_t q_stride,
                                     const void* k, int64_t k_stride,
                                     const void* w, int64_t w_stride,
                                     const float* bias, float scale, int dtype,
                                     int B, int Tq, int Tkv, int q_pos0, int H_I, int d_I,
                                     int k_sel, int32_t* indices, uint8_t* mask,
                                     uint32_t* bitmask, int64_t bitmask_words, void* stream);

/*
 * Sparse attention over a selection bitmask, on tcgen05 tensor cores.
 * Replaces _gather_along_seq + sparse_attention_ref (gsa_ref.py:185-238),
 * the Triton fused_sparse_attention (gsa_opt.py:349-383), and the output
 * gate apply (gsa_ref.py:177-180 / gsa_opt.py:700,720) when og != NULL:
 *
 *   o[b,r,h,:] = softmax_{j : bit(b,r,j)} (q[b,r,h,:].k[b,j,h,:] * scale) . v[b,j,h,:]
 *   out = og ? dtype(dtype(o) * dtype(sigmoid(og))) : dtype(o)
 *
 * A row with no selected key yields zeros (the reference's nan_to_num).
 *   q   [B, Tq, H*d]  row stride q_stride (bf16)
 *   k,v [B, Tkv, H*d] row strides k_stride, v_stride (bf16)
 *   bitmask [B, Tq, bitmask_words] uint32 as written by gsa_topk_select
 *   og  [B, Tq, H*d] output-gate logits (bias added), row stride og_stride, or NULL
 *   out [B, Tq, H*d] row stride out_stride (bf16)
 * Requires bf16, d == 128, 16-byte aligned rows, and a finite scale > 0
 * (GSA_ERR_INVALID_ARG otherwise).
 */
GSA_API int gsa_masked_attention(const void* q, int64_t q_stride,
                         const void* k, int64_t k_stride,
                         const void* v, int64_t v_stride,
                         const uint32_t* bitmask, int64_t bitmask_words,
                         const void* og, int64_t og_stride,
                         void* out, int64_t out_stride,
                         float scale, int B, int Tq, int Tkv, int q_pos0,
                         int H, int d, void* stream);

/*
 * Index-gather sparse attention (any index lists, duplicates allowed).
 * Replaces fused_sparse_attention (gsa_opt.py:349-383) / sparse_attention_ref
 * (gsa_ref.py:202-238) for explicit (indices, mask) inputs.  Indices are
 * clamped to [0, Tkv-1] as the reference does (gsa_ref.py:196); slots with
 * mask 0 are skipped; a row with no valid slot yields zeros.
 *   q [B, Tq, H, d], k/v [B, Tkv, H, d] with row strides (elements)
 *   indices [B, Tq, k_sel] int32, mask [B, Tq, k_sel] uint8 (NULL = all 1)
 *   out [B, Tq, H, d] row stride out_stride
 * bf16 or f32; d in {64, 128, 256}.
 */
GSA_API int gsa_gather_attention(const void* q, int64_t q_stride,
                         const void* k, int64_t k_stride,
                         const void* v, int64_t v_stride,
                         const int32_t* indices, const uint8_t* mask, int k_sel,
                         void* out, int64_t out_stride,
                         float scale, int dtype, int B, int Tq, int Tkv,
                         int H, int d, void* stream);

/*
 * Element-wise output gate (G1) without attention, for callers that run
 * gsa_gather_attention: out = dtype(o * dtype(sigmoid(og))).  Replaces
 * OutputGate.forward's sigmoid/multiply (gsa_ref.py:177-180).
 *   o, out [rows, width] with row strides; og [rows, width] row stride og_stride.
 */
GSA_API int gsa_output_gate(const void* o, int64_t o_stride,
                    const void* og, int64_t og_stride,
                    void* out, int64_t out_stride,
                    int dtype, int rows, int width, void* stream);

/*
 * Fused projection GEMM with RoPE and the value gate in its epilogue (bf16).
 * Replaces the mega-GEMM of gsa_opt.py:582-609 (torch.addmm over the
 * concatenated weights, biases added) together with the element-wise track_B
 * work after it (gsa_opt.py:683-696: value gate, RoPE on q and k):
 *
 *   q_out = RoPE(x Wq^T), k_out = RoPE(x Wk^T)          [M, D] contiguous
 *   v_out = (x Wv^T) * sigmoid(x Wvg^T + b_vg)            [M, D] contiguous
 *   rest  = og | iq | ik | iw = x [Wog; Wiq; Wik; Wiw]^T + [b_og; 0; 0; b_iw]
 *           [M, rest_stride], columns [0, D + H_I*d_I + d_I + H_I) written
 *
 * rounded to bf16 where the unfused torch ops round (each projection once,
 * then as gsa_rope_gates).  Row m (of M = B*T) has the rotary position
 * pos0 + m % T, i.e. row pos0 + m % T of the [table_rows, d] bf16 tables
 * cos / sin.  The weights come packed by gsa_fused_projection_pack:
 * w_packed [gsa_fused_projection_rows(D, H_I, d_I), D] bf16 and b_packed
 * float32 of the same row count.  Requires d == 128, D = H*d a multiple of
 * 256, 16-byte aligned rows, rest_stride >= gsa_fused_projection_rest_width.
 * One launch of a persistent tcgen05 kernel (clusters of two CTAs); the
 * accumulation order differs from cuBLAS's, so single outputs may differ from
 * the unfused path by one bf16 rounding step.  Allocates nothing.
 */
GSA_API int gsa_fused_projection(const void* x, int64_t x_stride,
                         const void* w_packed, const float* b_packed,
                         int M, int D, int H, int d, int H_I, int d_I,
                         int T, int pos0, const void* cos, const void* sin,
                         int64_t table_rows,
                         void* q_out, void* k_out, void* v_out,
                         void* rest, int64_t rest_stride, void* stream);

/* Rows of the packed weight (256 per column tile), 0 for unsupported sizes. */
GSA_API int64_t gsa_fused_projection_rows(int D, int H_I, int d_I);

/* Minimum rest_stride: D + H_I*d_I + d_I + H_I rounded up to 64. */
GSA_API int64_t gsa_fused_projection_rest_width(int D, int H_I, int d_I);

/*
 * Packs the module's projection weights for gsa_fused_projection (device
 * copies on `stream`; call again after the weights change).  Replaces
 * fuse_projections (gsa_opt.py:582-609) for this layout:
 *   w_q, w_k, w_v, w_vg, w_og [D, D]; w_iq [H_I*d_I, D]; w_ik [d_I, D];
 *   w_iw [H_I, D]: bf16, contiguous (nn.Linear.weight layout);
 *   b_vg, b_og [D], b_iw [H_I]: float32 (NULL = zero).
 * Output: w_packed [rows, D] bf16 and b_packed [rows] float32, rows =
 * gsa_fused_projection_rows(D, H_I, d_I).
 */
GSA_API int gsa_fused_projection_pack(const void* w_q, const void* w_k,
                         const void* w_v, const void* w_vg, const void* w_og,
                         const void* w_iq, const void* w_ik, const void* w_iw,
                         const float* b_vg, const float* b_og, const float* b_iw,
                         int D, int H_I, int d_I,
                         void* w_packed, float* b_packed, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GSA_B200_H_ */
