// topk.cu — per-row top-k selection over causal indexer scores.
//
// Replaces AdaptiveTopKSelector.forward (gsa_ref.py:138-150): k_eff largest
// of the row's valid scores (the reference maps -inf to -1e9 so valid
// scores always win), plus the ascending index sort of gsa_opt.py:674-677.
// Ties are broken toward the lower key index (torch.topk leaves tie order
// unspecified).
//
// One CTA per query row.  The row's valid scores (n = min(pos+1, Tkv)) are
// turned into order-preserving uint32 keys, staged in shared memory when
// they fit, and the k-th largest key is found by an MSB-first radix select
// (8-bit digits, warp-aggregated shared-memory histograms).  The select
// stops as soon as the bin holding the k-th key contains exactly the number
// of keys still needed.  A final pass in index order emits the selected
// columns in ascending order (block-wide ballots + scans) and writes one
// bitmask word per warp directly from the ballot.
#include "kernels.h"

namespace gsa {
namespace {

constexpr int kTopkThreads = 512;
constexpr int kTopkWarps = kTopkThreads / 32;
// Rows up to this many keys are staged in shared memory (160 KB).
constexpr int kTopkStageMax = 40960;

__device__ __forceinline__ uint32_t ord_key(float f) {
  const uint32_t x = __float_as_uint(f);
  return (x & 0x80000000u) ? ~x : (x | 0x80000000u);
}
// ord_key(-inf): 0xFF800000 inverted.
constexpr uint32_t kNegInfKey = 0x007FFFFFu;

template <bool STAGED>
__global__ void __launch_bounds__(kTopkThreads) topk_kernel(
    const float* __restrict__ scores, int64_t score_stride, int Tq, int Tkv, int q_pos0, int k_sel,
    int32_t* __restrict__ indices, uint8_t* __restrict__ mask, uint32_t* __restrict__ bitmask,
    int64_t bm_words) {
  extern __shared__ uint32_t skeys[];
  __shared__ int hist[256];
  __shared__ int warp_a[kTopkWarps];
  __shared__ int warp_b[kTopkWarps];
  __shared__ int sh_digit, sh_above, sh_bin;

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int64_t row = blockIdx.x;  // b * Tq + r
  const int r = static_cast<int>(row % Tq);
  const int pos = q_pos0 + r;
  const int n = min(pos + 1, Tkv);
  const float* srow = scores + row * score_stride;
  int32_t* irow = indices ? indices + row * k_sel : nullptr;
  uint8_t* mrow = mask ? mask + row * k_sel : nullptr;
  uint32_t* brow = bitmask ? bitmask + row * bm_words : nullptr;

  if (STAGED) {
    for (int j = tid; j < n; j += kTopkThreads) skeys[j] = ord_key(__ldg(srow + j));
    __syncthreads();
  }
  auto key_at = [&](int j) -> uint32_t {
    if (STAGED) return skeys[j];
    return ord_key(__ldg(srow + j));
  };

  // ---- radix select of the k-th largest key (MSB first, 8-bit digits).
  // With n <= k_sel every key is taken: prefix/pmask stay 0, so all keys
  // fall in the "equal" class and krem = k_sel >= n takes them all.
  uint32_t prefix = 0, pmask = 0;
  int krem = k_sel;  // keys still to take from the current prefix class
  for (int shift = 24; n > k_sel && shift >= 0; shift -= 8) {
    if (tid < 256) hist[tid] = 0;
    __syncthreads();
    for (int j0 = 0; j0 < n; j0 += kTopkThreads) {
      const int j = j0 + tid;
      const bool valid = j < n;
      const uint32_t u = valid ? key_at(j) : 0u;
      const bool in = valid && ((u & pmask) == prefix);
      const uint32_t digit = in ? ((u >> shift) & 255u) : 256u;
      const uint32_t peers = __match_any_sync(0xFFFFFFFFu, digit);
      if (in && lane == __ffs(peers) - 1) atomicAdd(&hist[digit], __popc(peers));
    }
    __syncthreads();
    // Inclusive scan of bins in descending digit order: thread t holds bin 255-t.
    int own = 0, cum = 0;
    if (tid < 256) {
      own = hist[255 - tid];
      cum = own;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xFFFFFFFFu, cum, o);
        if (lane >= o) cum += y;
      }
      if (lane == 31) warp_a[warp] = cum;
    }
    __syncthreads();
    if (tid < 256) {
      for (int w = 0; w < warp; ++w) cum += warp_a[w];
      if (cum >= krem && cum - own < krem) {
        sh_digit = 255 - tid;
        sh_above = cum - own;
        sh_bin = own;
      }
    }
    __syncthreads();
    prefix |= static_cast<uint32_t>(sh_digit) << shift;
    pmask |= 255u << shift;
    krem -= sh_above;
    const bool exact = (sh_bin == krem);
    __syncthreads();
    if (exact) break;
  }

  // ---- emit selected columns in ascending order; keys whose masked prefix
  // is above `prefix` are taken, those equal to it are taken lowest-index
  // first until krem are taken.  A selected column whose score is -inf is
  // listed with mask 0 and gets no bitmask bit (the reference's
  // `mask = gathered != -inf`).
  int base = 0, eq_taken = 0;
  const int span = ((n + 31) / 32) * 32;
  for (int j0 = 0; j0 < span; j0 += kTopkThreads) {
    const int j = j0 + tid;
    const bool valid = j < n;
    const uint32_t raw = valid ? key_at(j) : 0u;
    const uint32_t u = raw & pmask;
    const bool gt = valid && u > prefix;
    const bool eq = valid && u == prefix;
    const uint32_t lt_mask = (1u << lane) - 1u;
    const uint32_t eqb = __ballot_sync(0xFFFFFFFFu, eq);
    if (lane == 0) warp_a[warp] = __popc(eqb);
    __syncthreads();
    int eq_before = eq_taken + __popc(eqb & lt_mask);
    int eq_total = 0;
#pragma unroll
    for (int w = 0; w < kTopkWarps; ++w) {
      const int c = warp_a[w];
      if (w < warp) eq_before += c;
      eq_total += c;
    }
    const bool sel = gt || (eq && eq_before < krem);
    const uint32_t selb = __ballot_sync(0xFFFFFFFFu, sel);
    if (lane == 0) warp_b[warp] = __popc(selb);
    __syncthreads();
    int sel_before = base + __popc(selb & lt_mask);
    int sel_total = 0;
#pragma unroll
    for (int w = 0; w < kTopkWarps; ++w) {
      const int c = warp_b[w];
      if (w < warp) sel_before += c;
      sel_total += c;
    }
    const bool live = sel && raw != kNegInfKey;
    if (sel) {
      if (irow) irow[sel_before] = j;
      if (mrow) mrow[sel_before] = live ? 1 : 0;
    }
    const uint32_t liveb = __ballot_sync(0xFFFFFFFFu, live);
    const int64_t wd = (j0 >> 5) + warp;
    if (brow && lane == 0 && j0 + warp * 32 < span && wd < bm_words) brow[wd] = liveb;
    base += sel_total;
    eq_taken += eq_total;
    __syncthreads();
  }
  if (brow) {
    for (int64_t wd = span / 32 + tid; wd < bm_words; wd += kTopkThreads) brow[wd] = 0u;
  }
  // Filler slots past the selected ones (only when n < k_sel): future
  // positions, masked, as the reference's -inf picks.
  for (int s = base + tid; s < k_sel; s += kTopkThreads) {
    if (irow) irow[s] = min(s, Tkv - 1);
    if (mrow) mrow[s] = 0;
  }
}

}  // namespace

cudaError_t launch_topk(const float* scores, int64_t score_stride, int B, int Tq, int Tkv,
                        int q_pos0, int k_sel, int32_t* indices, uint8_t* mask, uint32_t* bitmask,
                        int64_t bitmask_words, cudaStream_t stream) {
  const int64_t rows = static_cast<int64_t>(B) * Tq;
  if (rows == 0) return cudaSuccess;
  const int max_n = min(q_pos0 + Tq, Tkv);
  if (max_n <= kTopkStageMax) {
    const size_t smem = static_cast<size_t>(max(max_n, 1)) * sizeof(uint32_t);
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr_set[dev]) {
      cudaError_t e = cudaFuncSetAttribute(topk_kernel<true>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           kTopkStageMax * static_cast<int>(sizeof(uint32_t)));
      if (e != cudaSuccess) return e;
      attr_set[dev] = true;
    }
    topk_kernel<true><<<static_cast<unsigned>(rows), kTopkThreads, smem, stream>>>(
        scores, score_stride, Tq, Tkv, q_pos0, k_sel, indices, mask, bitmask, bitmask_words);
  } else {
    topk_kernel<false><<<static_cast<unsigned>(rows), kTopkThreads, 0, stream>>>(
        scores, score_stride, Tq, Tkv, q_pos0, k_sel, indices, mask, bitmask, bitmask_words);
  }
  return cudaGetLastError();
}

}  // namespace gsa
