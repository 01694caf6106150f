// capi.cu — the extern "C" entry points of include/gsa_b200.h: argument
// checks, TMA tensor-map construction, dispatch to the kernels, status codes.
#include <cmath>
#include <cstdio>
#include <algorithm>
#include <cstring>
#include <atomic>
#include <mutex>

#include "kernels.h"

namespace {

constexpr int kVersion = 10000;  // 1.0.0
using gsa::kMaxDevices;

thread_local char g_last_error[256] = "";

// Device word that kernels set when a bounded wait expires.
__device__ int g_dev_err;

// Built-in scratch of gsa_indexer_topk_noalloc: the score rows that
// gsa_indexer_topk otherwise keeps in the caller's workspace.  Every GPU that
// loads the library holds it until the process exits.  In host code this name
// stands for the host-side shadow, not a device address: kernels receive the
// address that device_state() looks up per device.
static __device__ __align__(256) float g_noalloc_scratch[GSA_NOALLOC_SCRATCH_BYTES / sizeof(float)];

int set_cuda_error(cudaError_t e) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s: %s", cudaGetErrorName(e),
                cudaGetErrorString(e));
  return GSA_ERR_CUDA;
}

int set_error(int code, const char* what) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s", what);
  return code;
}

// Per-device state: sm_100 check result, the address of g_dev_err and the
// address of g_noalloc_scratch.  Filled once per device under g_dev_mu; `ready`
// is published with a release store after the other fields, so a thread that
// reads it true with an acquire load (outside the mutex) sees them filled.
struct DeviceState {
  std::atomic<bool> ready{false};
  bool sm100 = false;
  int* err = nullptr;
  float* noalloc = nullptr;
};
DeviceState g_dev[kMaxDevices];
std::mutex g_dev_mu;

int device_state(DeviceState** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error(e);
  if (dev < 0 || dev >= kMaxDevices) return set_error(GSA_ERR_NO_DEVICE, "device index out of range");
  DeviceState& st = g_dev[dev];
  if (!st.ready.load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(g_dev_mu);
    if (!st.ready.load(std::memory_order_relaxed)) {
      int major = 0;
      e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
      if (e != cudaSuccess) return set_cuda_error(e);
      st.sm100 = (major == 10);
      if (st.sm100) {
        // Both lookups need the library's module loaded on this device, which
        // only an sm_100 device can do (the library holds sm_100a code only).
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_dev_err);
        if (e != cudaSuccess) return set_cuda_error(e);
        st.err = static_cast<int*>(p);
        // The address of the built-in scratch of gsa_indexer_topk_noalloc on
        // this device (with this device current); the lookup allocates nothing.
        p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return set_cuda_error(e);
        st.noalloc = static_cast<float*>(p);
      }
      st.ready.store(true, std::memory_order_release);
    }
  }
  if (!st.sm100) return set_error(GSA_ERR_NO_DEVICE, "current device is not sm_100 (B200)");
  *out = &st;
  return GSA_OK;
}

// ---------------------------------------------------------------- TMA maps
typedef CUresult (*PFN_encodeTiled_t)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                      const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                      const cuuint32_t*, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion,
                                      CUtensorMapFloatOOBfill);

PFN_encodeTiled_t encode_fn() {
  static PFN_encodeTiled_t fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled_t>(p);
  });
  return fn;
}

// 3-D bf16 map over [z][y][x] with row stride `row_bytes` and batch stride
// `batch_bytes`; box {64, box_y, 1} with 128-byte swizzle; zero fill out of
// bounds.
int make_map_bf16_3d(CUtensorMap* map, const void* base, uint64_t x, uint64_t y, uint64_t z,
                     uint64_t row_bytes, uint64_t batch_bytes, uint32_t box_y) {
  PFN_encodeTiled_t fn = encode_fn();
  if (!fn) return set_error(GSA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[3] = {x, y, z};
  const cuuint64_t strides[2] = {row_bytes, batch_bytes};
  const cuuint32_t box[3] = {64, box_y, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    std::snprintf(g_last_error, sizeof(g_last_error), "cuTensorMapEncodeTiled failed (%d)",
                  static_cast<int>(r));
    return GSA_ERR_CUDA;
  }
  return GSA_OK;
}

// 3-D fp32 map of indexer score rows: [B][Tq][nkeys] with row stride
// `row_bytes`; box {16, 32, 1} with 64-byte swizzle (the layout the indexer
// epilogue stages), stores clipped past the last row and key.
int make_map_scores(CUtensorMap* map, float* base, uint64_t nkeys, uint64_t Tq, uint64_t B,
                    uint64_t row_bytes) {
  PFN_encodeTiled_t fn = encode_fn();
  if (!fn) return set_error(GSA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[3] = {nkeys, Tq, B};
  const cuuint64_t strides[2] = {row_bytes, row_bytes * Tq};
  const cuuint32_t box[3] = {16, 32, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    std::snprintf(g_last_error, sizeof(g_last_error), "cuTensorMapEncodeTiled failed (%d)",
                  static_cast<int>(r));
    return GSA_ERR_CUDA;
  }
  return GSA_OK;
}

// 2-D bf16 map over [rows][cols] with row stride `row_bytes`; box {64,
// box_rows} with 128-byte swizzle; loads fill zeros out of bounds, stores
// are clipped there.
int make_map_bf16_2d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows,
                     uint64_t row_bytes, uint32_t box_rows) {
  PFN_encodeTiled_t fn = encode_fn();
  if (!fn) return set_error(GSA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {64, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    std::snprintf(g_last_error, sizeof(g_last_error), "cuTensorMapEncodeTiled failed (%d)",
                  static_cast<int>(r));
    return GSA_ERR_CUDA;
  }
  return GSA_OK;
}

// Layout of the packed projection weight of gsa_fused_projection (the tile
// order proj_gemm.cu documents): q and k in D/256 tiles each, v/vg
// interleaved in D/128 tiles, then og | iq | ik | iw | zeros.
struct ProjLayout {
  int D, H_I, d_I;
  int64_t rest_cols() const { return D + static_cast<int64_t>(H_I) * d_I + d_I + H_I; }
  int q_tiles() const { return D / 256; }
  int v_tiles() const { return D / 128; }
  int rest_tiles() const { return static_cast<int>((rest_cols() + 255) / 256); }
  int n_tiles() const { return 2 * q_tiles() + v_tiles() + rest_tiles(); }
  int64_t rows() const { return static_cast<int64_t>(n_tiles()) * 256; }
  int64_t rest_width() const { return (rest_cols() + 63) / 64 * 64; }
  bool ok() const { return D > 0 && D % 256 == 0 && H_I > 0 && d_I > 0; }
};

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int finish(cudaError_t e) { return e == cudaSuccess ? GSA_OK : set_cuda_error(e); }

// The bf16 tensor-core indexer (indexer_tk.cu) covers H_I = 4, d_I = 64.
bool tc_path(int dtype, int H_I, int d_I) {
  return dtype == GSA_DTYPE_BF16 && H_I == 4 && d_I == 64;
}

// Tensor maps of the tensor-core indexer: q [B, Tq, 256] in boxes of 64 rows
// of one head; the launch's keys i = 0, 1, ... at sequence rows
// i * key_step + key_off of k [B, Tkv, 64], in boxes of 128 keys.
int make_tk_maps(CUtensorMap* qmap, CUtensorMap* kmap, const void* q, int64_t q_stride,
                 const void* k, int64_t k_stride, int B, int Tq, int Tkv, int key_step,
                 int key_off) {
  int rc = make_map_bf16_3d(qmap, q, 256, Tq, B, q_stride * 2,
                            static_cast<uint64_t>(Tq) * q_stride * 2,
                            gsa::indexer_tk_rows_per_cta());  // one box per head
  if (rc) return rc;
  const int nkeys = (Tkv - key_off + key_step - 1) / key_step;
  return make_map_bf16_3d(kmap, static_cast<const char*>(k) + static_cast<int64_t>(key_off) *
                                                                    k_stride * 2,
                          64, nkeys, B, static_cast<uint64_t>(key_step) * k_stride * 2,
                          static_cast<uint64_t>(Tkv) * k_stride * 2,
                          gsa::indexer_tk_keys_per_tile());
}

gsa::IndexerTkArgs tk_args(const void* w, int64_t w_stride, const float* bias, float scale, int B,
                           int Tq, int Tkv, int q_pos0, int* err) {
  gsa::IndexerTkArgs a{};
  a.w = w;
  a.w_stride = w_stride;
  a.bias = bias;
  a.scale = scale;
  a.B = B;
  a.Tq = Tq;
  a.Tkv = Tkv;
  a.q_pos0 = q_pos0;
  a.nkeys = Tkv;
  a.key_step = 1;
  a.key_off = 0;
  a.err = err;
  return a;
}

int indexer_impl(const void* q, int64_t q_stride, const void* k, int64_t k_stride, const void* w,
                 int64_t w_stride, const float* bias, float scale, int dtype, int B, int Tq,
                 int Tkv, int q_pos0, int H_I, int d_I, float* out, int64_t out_stride,
                 int fill_upper, cudaStream_t s) {
  if (dtype != GSA_DTYPE_BF16 && dtype != GSA_DTYPE_F32)
    return set_error(GSA_ERR_UNSUPPORTED, "dtype must be bf16 or f32");
  if (B < 0 || Tq < 0 || Tkv < 0 || q_pos0 < 0 || H_I <= 0 || d_I <= 0)
    return set_error(GSA_ERR_INVALID_ARG, "bad sizes");
  if (B == 0 || Tq == 0 || Tkv == 0) return GSA_OK;
  if (!q || !k || !w || !bias || !out) return set_error(GSA_ERR_INVALID_ARG, "null pointer");
  if (out_stride < Tkv) return set_error(GSA_ERR_INVALID_ARG, "out_stride < Tkv");
  if (q_stride < static_cast<int64_t>(H_I) * d_I || k_stride < d_I || w_stride < H_I)
    return set_error(GSA_ERR_INVALID_ARG, "row stride smaller than the row");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  if (fill_upper) {
    cudaError_t e = gsa::launch_fill_upper(out, out_stride, B, Tq, Tkv, q_pos0, s);
    if (e != cudaSuccess) return set_cuda_error(e);
  }
  if (tc_path(dtype, H_I, d_I)) {
    if (!aligned16(q) || !aligned16(k) || (q_stride * 2) % 16 || (k_stride * 2) % 16 ||
        !aligned16(out) || (out_stride * 4) % 16)
      return set_error(GSA_ERR_ALIGNMENT, "indexer rows must be 16-byte aligned");
    CUtensorMap qmap, kmap;
    rc = make_tk_maps(&qmap, &kmap, q, q_stride, k, k_stride, B, Tq, Tkv, 1, 0);
    if (rc) return rc;
    CUtensorMap omap;
    rc = make_map_scores(&omap, out, Tkv, Tq, B, out_stride * 4);
    if (rc) return rc;
    gsa::IndexerTkArgs a = tk_args(w, w_stride, bias, scale, B, Tq, Tkv, q_pos0, st->err);
    a.out = out;
    a.out_stride = out_stride;
    return finish(gsa::launch_indexer_tk(gsa::kIdxStore, qmap, kmap, omap, a, s));
  }
  if (H_I > 8 || d_I > 128 || H_I * d_I > 512)
    return set_error(GSA_ERR_UNSUPPORTED, "indexer heads/dims beyond the CUDA-core kernel");
  return finish(gsa::launch_indexer_simt(q, q_stride, k, k_stride, w, w_stride, bias, scale,
                                         dtype, B, Tq, Tkv, q_pos0, H_I, d_I, out, out_stride,
                                         s));
}


// Row stride (floats) of the score rows gsa_indexer_topk keeps in its workspace.
int64_t score_row_stride(int Tkv) { return (static_cast<int64_t>(Tkv) + 3) / 4 * 4; }

// The fused selection samples every kSampleStep-th key of a row to bracket
// its k-th score, kSampleZ standard deviations of the sample rank wide.
constexpr int kSampleStep = 8;
constexpr float kSampleZ = 4.0f;

// Selection state of one workspace row (stride words): the sure bits in the
// first gsa_bitmask_words(Tkv) words, one count per candidate list (two lists
// per indexer key chunk: the 16-key halves of its 32-key sub-tiles), then the
// lists, each of
// *per_list entries of two words, from word *cand_off on.  A list holds up to
// kMaxPerList candidates (nearly half of its 256 keys) where the row has room.
constexpr int kMaxPerList = 120;
void selection_layout(int Tkv, int64_t* cand_off, int* per_list) {
  const int64_t stride = score_row_stride(Tkv);
  const int64_t lists = 2 * ((static_cast<int64_t>(Tkv) + gsa::indexer_tk_keys_per_cta() - 1) /
                             gsa::indexer_tk_keys_per_cta());
  // lists start on 16-byte boundaries and hold an even number of entries: the
  // fix-up reads each with one bulk copy
  const int64_t off = (gsa_bitmask_words(Tkv) + lists + 3) / 4 * 4;
  *cand_off = off;
  *per_list =
      static_cast<int>(std::min<int64_t>(kMaxPerList, (stride - off) / (2 * lists))) & ~1;
}

// gsa_set_fused_selection's mode (GSA_FUSED_AUTO by default).
std::atomic<int> g_fused_mode{GSA_FUSED_AUTO};

// Where the fused selection applies at all: the tensor-core indexer, rows
// longer than twice k, at most kSelMaxKeys keys, room for the candidate lists.
bool fused_possible(int dtype, int H_I, int d_I, int Tkv, int k_sel) {
  if (!tc_path(dtype, H_I, d_I) || Tkv <= 2 * k_sel || Tkv < 4 * kSampleStep ||
      Tkv > gsa::kSelMaxKeys)
    return false;
  int64_t cand_off = 0;
  int per_list = 0;
  selection_layout(Tkv, &cand_off, &per_list);
  return per_list >= 8;
}

// The automatic choice takes the fused selection where it measured faster on
// B200: key ranges of at least kFusedMinRatio * k (T = 65536, k = 2048: 5.86
// against 6.59 ms for indexer + top-k; T = 16384: 0.52 against 0.51 ms;
// B = 8, T = 8192: 1.25 against 1.09 ms).
constexpr int kFusedMinRatio = 16;
bool fused_selection(int dtype, int H_I, int d_I, int Tkv, int k_sel) {
  const int mode = g_fused_mode.load(std::memory_order_relaxed);
  if (mode == GSA_FUSED_NEVER || !fused_possible(dtype, H_I, d_I, Tkv, k_sel)) return false;
  return mode == GSA_FUSED_ALWAYS ||
         static_cast<int64_t>(Tkv) >= static_cast<int64_t>(kFusedMinRatio) * k_sel;
}

int indexer_topk_fused(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                       const void* w, int64_t w_stride, const float* bias, float scale, int B,
                       int Tq, int Tkv, int q_pos0, int k_sel, float* ws, int32_t* indices,
                       uint8_t* mask, uint32_t* bitmask, int64_t bitmask_words, cudaStream_t s) {
  if (!aligned16(q) || !aligned16(k) || (q_stride * 2) % 16 || (k_stride * 2) % 16 ||
      !aligned16(ws))
    return set_error(GSA_ERR_ALIGNMENT, "indexer rows must be 16-byte aligned");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  const int64_t stride = score_row_stride(Tkv);
  const int64_t rows = static_cast<int64_t>(B) * Tq;
  gsa::SelectRowStats* stats = reinterpret_cast<gsa::SelectRowStats*>(ws + rows * stride);
  const int64_t sel_words = gsa_bitmask_words(Tkv);
  const int step = kSampleStep, off = kSampleStep - 1;
  int64_t cand_off = 0;
  int per_list = 0;
  selection_layout(Tkv, &cand_off, &per_list);
  CUtensorMap qmap, kmap, kmap_s, qmap_s;
  rc = make_tk_maps(&qmap, &kmap, q, q_stride, k, k_stride, B, Tq, Tkv, 1, 0);
  if (rc) return rc;
  rc = make_tk_maps(&qmap_s, &kmap_s, q, q_stride, k, k_stride, B, Tq, Tkv, step, off);
  if (rc) return rc;
  gsa::IndexerTkArgs a = tk_args(w, w_stride, bias, scale, B, Tq, Tkv, q_pos0, st->err);
  a.stats = stats;
  a.k_sel = k_sel;
  // 1. scores against every step-th key, into the rows' workspace
  gsa::IndexerTkArgs a1 = a;
  a1.nkeys = (Tkv - off + step - 1) / step;
  a1.key_step = step;
  a1.key_off = off;
  a1.out = ws;
  a1.out_stride = stride;
  CUtensorMap omap_s;
  rc = make_map_scores(&omap_s, ws, a1.nkeys, Tq, B, stride * 4);
  if (rc) return rc;
  cudaError_t e = gsa::launch_indexer_tk(gsa::kIdxSample, qmap_s, kmap_s, omap_s, a1, s);
  if (e != cudaSuccess) return set_cuda_error(e);
  // 2. per-row brackets [lo, hi] of the k-th score
  e = gsa::launch_select_threshold(ws, stride, B, Tq, Tkv, q_pos0, step, off, k_sel, kSampleZ,
                                   stats, s);
  if (e != cudaSuccess) return set_cuda_error(e);
  // 3. sure bits and candidates, over every key
  gsa::IndexerTkArgs a3 = a;
  a3.sel_bits = reinterpret_cast<uint32_t*>(ws);
  a3.sel_stride = stride;
  a3.bitmask_words = sel_words;
  a3.cand_off = cand_off;
  a3.cand_per_list = per_list;
  e = gsa::launch_indexer_tk(gsa::kIdxSelect, qmap, kmap, omap_s, a3, s);
  if (e != cudaSuccess) return set_cuda_error(e);
  // 4. full score rows of the rows whose bracket missed
  e = gsa::launch_select_scan(stats, B, Tq, Tkv, q_pos0, k_sel, gsa::indexer_tk_rows_per_cta(), s);
  if (e != cudaSuccess) return set_cuda_error(e);
  gsa::IndexerTkArgs a4 = a;
  a4.out = ws;
  a4.out_stride = stride;
  e = gsa::launch_indexer_tk(gsa::kIdxStoreFailed, qmap, kmap, omap_s, a4, s);
  if (e != cudaSuccess) return set_cuda_error(e);
  // 5. exact completion of every row
  return finish(gsa::launch_select_fixup(reinterpret_cast<const uint32_t*>(ws), stride, sel_words,
                                         cand_off, per_list, gsa::indexer_tk_keys_per_cta(),
                                         stats, B, Tq, Tkv, q_pos0, k_sel, indices, mask, bitmask,
                                         bitmask_words, st->err, s));
}

int indexer_topk_impl(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                      const void* w, int64_t w_stride, const float* bias, float scale, int dtype,
                      int B, int Tq, int Tkv, int q_pos0, int H_I, int d_I, int k_sel,
                      float* scores, int32_t* indices, uint8_t* mask, uint32_t* bitmask,
                      int64_t bitmask_words, cudaStream_t s) {
  if (fused_selection(dtype, H_I, d_I, Tkv, k_sel)) {
    if (!q || !k || !w || !bias) return set_error(GSA_ERR_INVALID_ARG, "null pointer");
    if (q_stride < static_cast<int64_t>(H_I) * d_I || k_stride < d_I || w_stride < H_I)
      return set_error(GSA_ERR_INVALID_ARG, "row stride smaller than the row");
    return indexer_topk_fused(q, q_stride, k, k_stride, w, w_stride, bias, scale, B, Tq, Tkv,
                              q_pos0, k_sel, scores, indices, mask, bitmask, bitmask_words, s);
  }
  const int64_t stride = score_row_stride(Tkv);
  int rc = indexer_impl(q, q_stride, k, k_stride, w, w_stride, bias, scale, dtype, B, Tq, Tkv,
                        q_pos0, H_I, d_I, scores, stride, 0, s);
  if (rc) return rc;
  // the indexer writes finite scores into every valid column
  return finish(gsa::launch_topk(scores, stride, B, Tq, Tkv, q_pos0, k_sel, k_sel,
                                 gsa::AdaptiveK{}, indices, mask, bitmask, bitmask_words,
                                 /*finite_rows=*/true, s));
}

// Adaptive-k workspace: the score rows, then row_var [B*Tq] floats, then the
// double var_sum on a 16-byte boundary.
int64_t adaptive_var_offset(int B, int Tq, int Tkv) {
  return static_cast<int64_t>(B) * Tq * score_row_stride(Tkv) * static_cast<int64_t>(sizeof(float));
}
int64_t adaptive_sum_offset(int B, int Tq, int Tkv) {
  const int64_t end = adaptive_var_offset(B, Tq, Tkv) +
                      static_cast<int64_t>(B) * Tq * static_cast<int64_t>(sizeof(float));
  return (end + 15) / 16 * 16;
}

int check_adaptive_k(int k_base, int k_min, int k_max) {
  if (k_base < 0 || k_min < 0 || k_max < 1 || k_min > k_max)
    return set_error(GSA_ERR_INVALID_ARG, "adaptive k needs k_base >= 0, 0 <= k_min <= k_max, "
                                          "k_max >= 1");
  return GSA_OK;
}

}  // namespace

extern "C" {

int gsa_version(void) { return kVersion; }

int gsa_set_fused_selection(int mode) {
  if (mode != GSA_FUSED_AUTO && mode != GSA_FUSED_ALWAYS && mode != GSA_FUSED_NEVER)
    return set_error(GSA_ERR_INVALID_ARG, "mode must be GSA_FUSED_AUTO, _ALWAYS or _NEVER");
  g_fused_mode.store(mode, std::memory_order_relaxed);
  return GSA_OK;
}

const char* gsa_status_string(int status) {
  switch (status) {
    case GSA_OK: return "ok";
    case GSA_ERR_INVALID_ARG: return "invalid argument";
    case GSA_ERR_ALIGNMENT: return "pointer or stride not 16-byte aligned";
    case GSA_ERR_UNSUPPORTED: return "unsupported shape or dtype";
    case GSA_ERR_CUDA: return "CUDA error";
    case GSA_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    case GSA_ERR_NO_DEVICE: return "no usable sm_100 device";
    default: return "unknown status";
  }
}

const char* gsa_last_error_string(void) { return g_last_error; }

int gsa_device_error(int* out, int reset) {
  if (!out) return set_error(GSA_ERR_INVALID_ARG, "out is NULL");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return set_cuda_error(e);
  e = cudaMemcpy(out, st->err, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return set_cuda_error(e);
  if (reset) {
    e = cudaMemset(st->err, 0, sizeof(int));
    if (e != cudaSuccess) return set_cuda_error(e);
  }
  return GSA_OK;
}

int64_t gsa_bitmask_words(int Tkv) {
  if (Tkv <= 0) return 0;
  return 4 * ((static_cast<int64_t>(Tkv) + 127) / 128);
}

int gsa_rope_gates(const void* q_src, const void* k_src, const void* v_src, const void* vg_src,
                   int64_t src_stride, int dtype, int B, int T, int H, int d, const void* cos,
                   const void* sin, void* q_out, void* k_out, void* v_out, void* stream) {
  if (dtype != GSA_DTYPE_BF16 && dtype != GSA_DTYPE_F32)
    return set_error(GSA_ERR_UNSUPPORTED, "dtype must be bf16 or f32");
  if (B < 0 || T < 0 || H <= 0 || d <= 0) return set_error(GSA_ERR_INVALID_ARG, "bad sizes");
  if (d % 16 != 0) return set_error(GSA_ERR_UNSUPPORTED, "d must be a multiple of 16");
  if (B == 0 || T == 0) return GSA_OK;
  if (!q_src || !k_src || !cos || !sin || !q_out || !k_out)
    return set_error(GSA_ERR_INVALID_ARG, "null pointer");
  if ((v_src == nullptr) != (vg_src == nullptr) || (v_src && !v_out))
    return set_error(GSA_ERR_INVALID_ARG, "v_src, vg_src and v_out go together");
  const int es = dtype == GSA_DTYPE_BF16 ? 2 : 4;
  const int64_t width = static_cast<int64_t>(H) * d;
  if (src_stride < width) return set_error(GSA_ERR_INVALID_ARG, "src_stride < H*d");
  if ((src_stride * es) % 16 || !aligned16(q_src) || !aligned16(k_src) ||
      (v_src && (!aligned16(v_src) || !aligned16(vg_src) || !aligned16(v_out))) ||
      !aligned16(cos) || !aligned16(sin) || !aligned16(q_out) || !aligned16(k_out))
    return set_error(GSA_ERR_ALIGNMENT, "rows must be 16-byte aligned");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  return finish(gsa::launch_rope_gates(q_src, k_src, v_src, vg_src, src_stride, dtype, B, T, H, d,
                                       cos, sin, q_out, k_out, v_out,
                                       static_cast<cudaStream_t>(stream)));
}

int gsa_indexer_scores(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                       const void* w, int64_t w_stride, const float* bias, float scale, int dtype,
                       int B, int Tq, int Tkv, int q_pos0, int H_I, int d_I, float* out,
                       int64_t out_stride, int fill_upper, void* stream) {
  return indexer_impl(q, q_stride, k, k_stride, w, w_stride, bias, scale, dtype, B, Tq, Tkv,
                      q_pos0, H_I, d_I, out, out_stride, fill_upper,
                      static_cast<cudaStream_t>(stream));
}

int64_t gsa_indexer_topk_workspace_size(int B, int Tq, int Tkv) {
  if (B <= 0 || Tq <= 0 || Tkv <= 0) return 0;
  return static_cast<int64_t>(B) * Tq *
         (score_row_stride(Tkv) * static_cast<int64_t>(sizeof(float)) +
          static_cast<int64_t>(sizeof(gsa::SelectRowStats)));
}

int gsa_indexer_topk(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                     const void* w, int64_t w_stride, const float* bias, float scale, int dtype,
                     int B, int Tq, int Tkv, int q_pos0, int H_I, int d_I, int k_sel,
                     void* workspace, int64_t workspace_bytes, int32_t* indices, uint8_t* mask,
                     uint32_t* bitmask, int64_t bitmask_words, void* stream) {
  if (B < 0 || Tq < 0 || Tkv <= 0 || q_pos0 < 0 || k_sel <= 0 || k_sel > Tkv)
    return set_error(GSA_ERR_INVALID_ARG, "bad sizes (need 0 < k_sel <= Tkv)");
  if (B == 0 || Tq == 0) return GSA_OK;
  if (!workspace) return set_error(GSA_ERR_INVALID_ARG, "workspace is NULL");
  if (workspace_bytes < gsa_indexer_topk_workspace_size(B, Tq, Tkv))
    return set_error(GSA_ERR_INVALID_ARG, "workspace smaller than gsa_indexer_topk_workspace_size");
  if (bitmask && bitmask_words < gsa_bitmask_words(Tkv))
    return set_error(GSA_ERR_INVALID_ARG, "bitmask_words < gsa_bitmask_words(Tkv)");
  return indexer_topk_impl(q, q_stride, k, k_stride, w, w_stride, bias, scale, dtype, B, Tq, Tkv,
                           q_pos0, H_I, d_I, k_sel, static_cast<float*>(workspace), indices, mask,
                           bitmask, bitmask_words, static_cast<cudaStream_t>(stream));
}

int gsa_indexer_topk_noalloc(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                             const void* w, int64_t w_stride, const float* bias, float scale,
                             int dtype, int B, int Tq, int Tkv, int q_pos0, int H_I, int d_I,
                             int k_sel, int32_t* indices, uint8_t* mask, uint32_t* bitmask,
                             int64_t bitmask_words, void* stream) {
  if (B < 0 || Tq < 0 || Tkv <= 0 || q_pos0 < 0 || k_sel <= 0 || k_sel > Tkv)
    return set_error(GSA_ERR_INVALID_ARG, "bad sizes (need 0 < k_sel <= Tkv)");
  if (B == 0 || Tq == 0) return GSA_OK;
  const int64_t need = gsa_indexer_topk_workspace_size(B, Tq, Tkv);
  if (need > static_cast<int64_t>(GSA_NOALLOC_SCRATCH_BYTES)) {
    std::snprintf(g_last_error, sizeof(g_last_error),
                  "gsa_indexer_topk_noalloc needs %lld bytes of scratch, more than its built-in "
                  "%lld; call gsa_indexer_topk with a workspace instead",
                  static_cast<long long>(need), static_cast<long long>(GSA_NOALLOC_SCRATCH_BYTES));
    return GSA_ERR_UNSUPPORTED;
  }
  if (bitmask && bitmask_words < gsa_bitmask_words(Tkv))
    return set_error(GSA_ERR_INVALID_ARG, "bitmask_words < gsa_bitmask_words(Tkv)");
  DeviceState* st = nullptr;
  int rc = device_state(&st);  // GSA_ERR_NO_DEVICE on anything but sm_100
  if (rc) return rc;
  return indexer_topk_impl(q, q_stride, k, k_stride, w, w_stride, bias, scale, dtype, B, Tq, Tkv,
                           q_pos0, H_I, d_I, k_sel, st->noalloc, indices, mask, bitmask,
                           bitmask_words, static_cast<cudaStream_t>(stream));
}

int gsa_topk_select(const float* scores, int64_t score_stride, int B, int Tq, int Tkv, int q_pos0,
                    int k_sel, int32_t* indices, uint8_t* mask, uint32_t* bitmask,
                    int64_t bitmask_words, void* stream) {
  if (B < 0 || Tq < 0 || Tkv <= 0 || q_pos0 < 0 || k_sel <= 0 || k_sel > Tkv)
    return set_error(GSA_ERR_INVALID_ARG, "bad sizes (need 0 < k_sel <= Tkv)");
  if (B == 0 || Tq == 0) return GSA_OK;
  if (!scores) return set_error(GSA_ERR_INVALID_ARG, "scores is NULL");
  if (score_stride < Tkv) return set_error(GSA_ERR_INVALID_ARG, "score_stride < Tkv");
  if (bitmask && bitmask_words < gsa_bitmask_words(Tkv))
    return set_error(GSA_ERR_INVALID_ARG, "bitmask_words < gsa_bitmask_words(Tkv)");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  return finish(gsa::launch_topk(scores, score_stride, B, Tq, Tkv, q_pos0, k_sel, k_sel,
                                 gsa::AdaptiveK{}, indices, mask, bitmask, bitmask_words,
                                 /*finite_rows=*/false, static_cast<cudaStream_t>(stream)));
}

int gsa_row_variance(const float* scores, int64_t score_stride, int B, int Tq, int Tkv,
                     int q_pos0, float* row_var, double* var_sum, void* stream) {
  if (B < 0 || Tq < 0 || Tkv <= 0 || q_pos0 < 0) return set_error(GSA_ERR_INVALID_ARG, "bad sizes");
  if (!row_var || !var_sum) return set_error(GSA_ERR_INVALID_ARG, "row_var / var_sum is NULL");
  if (reinterpret_cast<uintptr_t>(var_sum) % alignof(double))
    return set_error(GSA_ERR_ALIGNMENT, "var_sum must be 8-byte aligned");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (B == 0 || Tq == 0) return finish(cudaMemsetAsync(var_sum, 0, sizeof(double), s));
  if (!scores) return set_error(GSA_ERR_INVALID_ARG, "scores is NULL");
  if (score_stride < Tkv) return set_error(GSA_ERR_INVALID_ARG, "score_stride < Tkv");
  return finish(gsa::launch_row_variance(scores, score_stride, B, Tq, Tkv, q_pos0, row_var,
                                         var_sum, s));
}

namespace {
int topk_select_adaptive_impl(const float* scores, int64_t score_stride, int B, int Tq, int Tkv,
                              int q_pos0, int k_base, int k_min, int k_max, const float* row_var,
                              const double* var_sum, int64_t var_rows, int32_t* row_k,
                              int32_t* indices, uint8_t* mask, uint32_t* bitmask,
                              int64_t bitmask_words, bool finite_rows, void* stream) {
  if (B < 0 || Tq < 0 || Tkv <= 0 || q_pos0 < 0) return set_error(GSA_ERR_INVALID_ARG, "bad sizes");
  int rc = check_adaptive_k(k_base, k_min, k_max);
  if (rc) return rc;
  if (B == 0 || Tq == 0) return GSA_OK;
  if (!scores || !row_var || !var_sum)
    return set_error(GSA_ERR_INVALID_ARG, "scores / row_var / var_sum is NULL");
  if (var_rows < 1) return set_error(GSA_ERR_INVALID_ARG, "var_rows < 1");
  if (score_stride < Tkv) return set_error(GSA_ERR_INVALID_ARG, "score_stride < Tkv");
  if (bitmask && bitmask_words < gsa_bitmask_words(Tkv))
    return set_error(GSA_ERR_INVALID_ARG, "bitmask_words < gsa_bitmask_words(Tkv)");
  DeviceState* st = nullptr;
  rc = device_state(&st);
  if (rc) return rc;
  gsa::AdaptiveK ad;
  ad.row_var = row_var;
  ad.var_sum = var_sum;
  ad.var_rows = var_rows;
  ad.k_base = k_base;
  ad.k_min = k_min;
  ad.k_max = k_max;
  ad.row_k = row_k;
  const int width = gsa_adaptive_k_width(k_max, Tkv);
  return finish(gsa::launch_topk(scores, score_stride, B, Tq, Tkv, q_pos0, 0, width, ad, indices,
                                 mask, bitmask, bitmask_words, finite_rows,
                                 static_cast<cudaStream_t>(stream)));
}
}  // namespace

int gsa_topk_select_adaptive(const float* scores, int64_t score_stride, int B, int Tq, int Tkv,
                             int q_pos0, int k_base, int k_min, int k_max, const float* row_var,
                             const double* var_sum, int64_t var_rows, int32_t* row_k,
                             int32_t* indices, uint8_t* mask, uint32_t* bitmask,
                             int64_t bitmask_words, void* stream) {
  return topk_select_adaptive_impl(scores, score_stride, B, Tq, Tkv, q_pos0, k_base, k_min,
                                   k_max, row_var, var_sum, var_rows, row_k, indices, mask,
                                   bitmask, bitmask_words, /*finite_rows=*/false, stream);
}

int gsa_adaptive_k_width(int k_max, int Tkv) { return k_max < Tkv ? k_max : Tkv; }

int64_t gsa_indexer_topk_adaptive_workspace_size(int B, int Tq, int Tkv) {
  if (B <= 0 || Tq <= 0 || Tkv <= 0) return 0;
  return adaptive_sum_offset(B, Tq, Tkv) + 16;
}

int gsa_indexer_topk_adaptive(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                              const void* w, int64_t w_stride, const float* bias, float scale,
                              int dtype, int B, int Tq, int Tkv, int q_pos0, int H_I, int d_I,
                              int k_base, int k_min, int k_max, void* workspace,
                              int64_t workspace_bytes, int32_t* row_k, int32_t* indices,
                              uint8_t* mask, uint32_t* bitmask, int64_t bitmask_words,
                              void* stream) {
  if (B < 0 || Tq < 0 || Tkv <= 0 || q_pos0 < 0) return set_error(GSA_ERR_INVALID_ARG, "bad sizes");
  int rc = check_adaptive_k(k_base, k_min, k_max);
  if (rc) return rc;
  if (B == 0 || Tq == 0) return GSA_OK;
  if (!workspace) return set_error(GSA_ERR_INVALID_ARG, "workspace is NULL");
  if (workspace_bytes < gsa_indexer_topk_adaptive_workspace_size(B, Tq, Tkv))
    return set_error(GSA_ERR_INVALID_ARG,
                     "workspace smaller than gsa_indexer_topk_adaptive_workspace_size");
  if (!aligned16(workspace)) return set_error(GSA_ERR_ALIGNMENT, "workspace not 16-byte aligned");
  if (bitmask && bitmask_words < gsa_bitmask_words(Tkv))
    return set_error(GSA_ERR_INVALID_ARG, "bitmask_words < gsa_bitmask_words(Tkv)");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* base = static_cast<char*>(workspace);
  float* scores = reinterpret_cast<float*>(base);
  float* row_var = reinterpret_cast<float*>(base + adaptive_var_offset(B, Tq, Tkv));
  double* var_sum = reinterpret_cast<double*>(base + adaptive_sum_offset(B, Tq, Tkv));
  const int64_t stride = score_row_stride(Tkv);
  rc = indexer_impl(q, q_stride, k, k_stride, w, w_stride, bias, scale, dtype, B, Tq, Tkv, q_pos0,
                    H_I, d_I, scores, stride, 0, s);
  if (rc) return rc;
  rc = gsa_row_variance(scores, stride, B, Tq, Tkv, q_pos0, row_var, var_sum, stream);
  if (rc) return rc;
  return topk_select_adaptive_impl(scores, stride, B, Tq, Tkv, q_pos0, k_base, k_min, k_max,
                                   row_var, var_sum, static_cast<int64_t>(B) * Tq, row_k, indices,
                                   mask, bitmask, bitmask_words, /*finite_rows=*/true, stream);
}

int gsa_masked_attention(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                         const void* v, int64_t v_stride, const uint32_t* bitmask,
                         int64_t bitmask_words, const void* og, int64_t og_stride, void* out,
                         int64_t out_stride, float scale, int B, int Tq, int Tkv, int q_pos0,
                         int H, int d, void* stream) {
  if (B < 0 || Tq < 0 || Tkv < 0 || q_pos0 < 0 || H <= 0 || d <= 0)
    return set_error(GSA_ERR_INVALID_ARG, "bad sizes");
  if (d != 128) return set_error(GSA_ERR_UNSUPPORTED, "masked attention needs d == 128");
  if (!(scale > 0.f) || !std::isfinite(scale))  // the lazy running max assumes scale > 0
    return set_error(GSA_ERR_INVALID_ARG, "masked attention needs a finite scale > 0");
  if (B == 0 || Tq == 0 || Tkv == 0) return GSA_OK;
  if (!q || !k || !v || !bitmask || !out) return set_error(GSA_ERR_INVALID_ARG, "null pointer");
  const int64_t width = static_cast<int64_t>(H) * d;
  if (q_stride < width || k_stride < width || v_stride < width || out_stride < width ||
      (og && og_stride < width))
    return set_error(GSA_ERR_INVALID_ARG, "row stride smaller than H*d");
  if (bitmask_words < gsa_bitmask_words(Tkv) || bitmask_words % 4)
    return set_error(GSA_ERR_INVALID_ARG, "bitmask_words must be >= gsa_bitmask_words(Tkv), %4");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || !aligned16(bitmask) ||
      (og && !aligned16(og)) || (q_stride * 2) % 16 || (k_stride * 2) % 16 ||
      (v_stride * 2) % 16 || (out_stride * 2) % 16 || (og && (og_stride * 2) % 16))
    return set_error(GSA_ERR_ALIGNMENT, "attention rows must be 16-byte aligned");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  CUtensorMap qmap, kmap, vmap;
  rc = make_map_bf16_3d(&qmap, q, width, Tq, B, q_stride * 2,
                        static_cast<uint64_t>(Tq) * q_stride * 2, 128);
  if (rc) return rc;
  rc = make_map_bf16_3d(&kmap, k, width, Tkv, B, k_stride * 2,
                        static_cast<uint64_t>(Tkv) * k_stride * 2, 128);
  if (rc) return rc;
  rc = make_map_bf16_3d(&vmap, v, width, Tkv, B, v_stride * 2,
                        static_cast<uint64_t>(Tkv) * v_stride * 2, 128);
  if (rc) return rc;
  gsa::MaskedAttnArgs a;
  a.bitmask = bitmask;
  a.bitmask_words = bitmask_words;
  a.og = og;
  a.og_stride = og_stride;
  a.out = out;
  a.out_stride = out_stride;
  a.scale = scale;
  a.B = B;
  a.Tq = Tq;
  a.Tkv = Tkv;
  a.q_pos0 = q_pos0;
  a.H = H;
  a.err = st->err;
  int expected = 0;
  const int regs = gsa::masked_attention_regs(&expected);
  if (regs != expected) {
    std::snprintf(g_last_error, sizeof(g_last_error),
                  "masked_attn_kernel was built with %d registers per thread; its setmaxnreg "
                  "split needs %d",
                  regs, expected);
    return GSA_ERR_UNSUPPORTED;
  }
  return finish(gsa::launch_masked_attention(qmap, kmap, vmap, a, static_cast<cudaStream_t>(stream)));
}

int gsa_gather_attention(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                         const void* v, int64_t v_stride, const int32_t* indices,
                         const uint8_t* mask, int k_sel, void* out, int64_t out_stride,
                         float scale, int dtype, int B, int Tq, int Tkv, int H, int d,
                         void* stream) {
  if (dtype != GSA_DTYPE_BF16 && dtype != GSA_DTYPE_F32)
    return set_error(GSA_ERR_UNSUPPORTED, "dtype must be bf16 or f32");
  if (B < 0 || Tq < 0 || Tkv <= 0 || H <= 0 || k_sel < 0)
    return set_error(GSA_ERR_INVALID_ARG, "bad sizes");
  if (d != 64 && d != 128 && d != 256) return set_error(GSA_ERR_UNSUPPORTED, "d must be 64/128/256");
  if (B == 0 || Tq == 0) return GSA_OK;
  if (!q || !k || !v || !out || (k_sel > 0 && !indices))
    return set_error(GSA_ERR_INVALID_ARG, "null pointer");
  const int64_t width = static_cast<int64_t>(H) * d;
  if (q_stride < width || k_stride < width || v_stride < width || out_stride < width)
    return set_error(GSA_ERR_INVALID_ARG, "row stride smaller than H*d");
  const int es = dtype == GSA_DTYPE_BF16 ? 2 : 4;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) ||
      (q_stride * es) % 16 || (k_stride * es) % 16 || (v_stride * es) % 16 ||
      (out_stride * es) % 16)
    return set_error(GSA_ERR_ALIGNMENT, "attention rows must be 16-byte aligned");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  return finish(gsa::launch_gather_attention(q, q_stride, k, k_stride, v, v_stride, indices, mask,
                                             k_sel, out, out_stride, scale, dtype, B, Tq, Tkv, H,
                                             d, static_cast<cudaStream_t>(stream)));
}

int gsa_output_gate(const void* o, int64_t o_stride, const void* og, int64_t og_stride, void* out,
                    int64_t out_stride, int dtype, int rows, int width, void* stream) {
  if (dtype != GSA_DTYPE_BF16 && dtype != GSA_DTYPE_F32)
    return set_error(GSA_ERR_UNSUPPORTED, "dtype must be bf16 or f32");
  if (rows < 0 || width < 0) return set_error(GSA_ERR_INVALID_ARG, "bad sizes");
  if (width % 8) return set_error(GSA_ERR_UNSUPPORTED, "width must be a multiple of 8");
  if (rows == 0 || width == 0) return GSA_OK;
  if (!o || !og || !out) return set_error(GSA_ERR_INVALID_ARG, "null pointer");
  const int es = dtype == GSA_DTYPE_BF16 ? 2 : 4;
  if (!aligned16(o) || !aligned16(og) || !aligned16(out) || (o_stride * es) % 16 ||
      (og_stride * es) % 16 || (out_stride * es) % 16)
    return set_error(GSA_ERR_ALIGNMENT, "rows must be 16-byte aligned");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  return finish(gsa::launch_output_gate(o, o_stride, og, og_stride, out, out_stride, dtype, rows,
                                        width, static_cast<cudaStream_t>(stream)));
}

int64_t gsa_fused_projection_rows(int D, int H_I, int d_I) {
  const ProjLayout L{D, H_I, d_I};
  return L.ok() ? L.rows() : 0;
}

int64_t gsa_fused_projection_rest_width(int D, int H_I, int d_I) {
  const ProjLayout L{D, H_I, d_I};
  return L.ok() ? L.rest_width() : 0;
}

int gsa_fused_projection_pack(const void* w_q, const void* w_k, const void* w_v, const void* w_vg,
                              const void* w_og, const void* w_iq, const void* w_ik,
                              const void* w_iw, const float* b_vg, const float* b_og,
                              const float* b_iw, int D, int H_I, int d_I, void* w_packed,
                              float* b_packed, void* stream) {
  const ProjLayout L{D, H_I, d_I};
  if (!L.ok())
    return set_error(GSA_ERR_UNSUPPORTED, "D must be a positive multiple of 256, H_I, d_I > 0");
  if (!w_q || !w_k || !w_v || !w_vg || !w_og || !w_iq || !w_ik || !w_iw || !w_packed || !b_packed)
    return set_error(GSA_ERR_INVALID_ARG, "null pointer");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t row = static_cast<size_t>(D) * 2;
  char* wp = static_cast<char*>(w_packed);
  cudaError_t e = cudaSuccess;
  auto rows_to = [&](int64_t dst_row, const void* src, int64_t src_row, int64_t n) {
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(wp + dst_row * row, static_cast<const char*>(src) + src_row * row,
                          n * row, cudaMemcpyDeviceToDevice, s);
  };
  auto bias_to = [&](int64_t dst, const float* src, int64_t src_off, int64_t n) {
    if (e == cudaSuccess && src)
      e = cudaMemcpyAsync(b_packed + dst, src + src_off, n * sizeof(float),
                          cudaMemcpyDeviceToDevice, s);
  };
  rows_to(0, w_q, 0, D);
  rows_to(D, w_k, 0, D);
  if (e == cudaSuccess) e = cudaMemsetAsync(b_packed, 0, L.rows() * sizeof(float), s);
  for (int i = 0; i < D / 128; ++i) {
    const int64_t t0 = 2 * static_cast<int64_t>(D) + 256 * i;
    rows_to(t0, w_v, 128 * i, 128);
    rows_to(t0 + 128, w_vg, 128 * i, 128);
    bias_to(t0 + 128, b_vg, 128 * i, 128);
  }
  int64_t r = 4 * static_cast<int64_t>(D);
  rows_to(r, w_og, 0, D);
  bias_to(r, b_og, 0, D);
  r += D;
  rows_to(r, w_iq, 0, static_cast<int64_t>(H_I) * d_I);
  r += static_cast<int64_t>(H_I) * d_I;
  rows_to(r, w_ik, 0, d_I);
  r += d_I;
  rows_to(r, w_iw, 0, H_I);
  bias_to(r, b_iw, 0, H_I);
  r += H_I;
  if (e == cudaSuccess) e = cudaMemsetAsync(wp + r * row, 0, (L.rows() - r) * row, s);
  return finish(e);
}

int gsa_fused_projection(const void* x, int64_t x_stride, const void* w_packed,
                         const float* b_packed, int M, int D, int H, int d, int H_I, int d_I,
                         int T, int pos0, const void* cos, const void* sin, int64_t table_rows,
                         void* q_out, void* k_out, void* v_out, void* rest, int64_t rest_stride,
                         void* stream) {
  const ProjLayout L{D, H_I, d_I};
  if (M < 0 || H <= 0 || d <= 0 || T <= 0 || pos0 < 0 || table_rows < 0)
    return set_error(GSA_ERR_INVALID_ARG, "bad sizes");
  if (d != 128 || static_cast<int64_t>(H) * d != D || !L.ok())
    return set_error(GSA_ERR_UNSUPPORTED, "needs d == 128, D == H*d, D a multiple of 256");
  if (M == 0) return GSA_OK;
  if (!x || !w_packed || !b_packed || !cos || !sin || !q_out || !k_out || !v_out || !rest)
    return set_error(GSA_ERR_INVALID_ARG, "null pointer");
  if (x_stride < D || rest_stride < L.rest_width())
    return set_error(GSA_ERR_INVALID_ARG, "x_stride < D or rest_stride < the rest width");
  if (table_rows < static_cast<int64_t>(pos0) + std::min(T, M))
    return set_error(GSA_ERR_INVALID_ARG, "rotary tables end before the last position");
  if (!aligned16(x) || (x_stride * 2) % 16 || !aligned16(w_packed) || !aligned16(b_packed) ||
      !aligned16(cos) || !aligned16(sin) || !aligned16(q_out) || !aligned16(k_out) ||
      !aligned16(v_out) || !aligned16(rest) || (rest_stride * 2) % 16)
    return set_error(GSA_ERR_ALIGNMENT, "rows must be 16-byte aligned");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  int clusters = gsa::proj_gemm_max_clusters();
  if (clusters <= 0) return set_error(GSA_ERR_CUDA, "no two-CTA cluster fits this device");
  CUtensorMap xmap, wmap, qmap, kmap, vmap, rmap;
  if ((rc = make_map_bf16_2d(&xmap, x, D, M, x_stride * 2, 128))) return rc;
  if ((rc = make_map_bf16_2d(&wmap, w_packed, D, L.rows(), static_cast<uint64_t>(D) * 2, 128)))
    return rc;
  if ((rc = make_map_bf16_2d(&qmap, q_out, D, M, static_cast<uint64_t>(D) * 2, 32))) return rc;
  if ((rc = make_map_bf16_2d(&kmap, k_out, D, M, static_cast<uint64_t>(D) * 2, 32))) return rc;
  if ((rc = make_map_bf16_2d(&vmap, v_out, D, M, static_cast<uint64_t>(D) * 2, 32))) return rc;
  if ((rc = make_map_bf16_2d(&rmap, rest, L.rest_width(), M, rest_stride * 2, 32))) return rc;
  gsa::ProjGemmArgs a{};
  a.M = M;
  a.K = D;
  a.n_tiles = L.n_tiles();
  a.q_tiles = L.q_tiles();
  a.v_tiles = L.v_tiles();
  a.rest_boxes = static_cast<int>(L.rest_width() / 64);
  a.T = T;
  a.pos0 = pos0;
  a.cos = static_cast<const __nv_bfloat16*>(cos);
  a.sin = static_cast<const __nv_bfloat16*>(sin);
  a.bias = b_packed;
  a.err = st->err;
  const int64_t tiles = (static_cast<int64_t>(M) + 255) / 256 * L.n_tiles();
  clusters = static_cast<int>(std::min<int64_t>(clusters, tiles));
  return finish(gsa::launch_proj_gemm(xmap, wmap, qmap, kmap, vmap, rmap, a, clusters,
                                      static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
