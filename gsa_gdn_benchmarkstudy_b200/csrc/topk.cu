// topk.cu — per-row top-k selection over causal indexer scores.
//
// Replaces AdaptiveTopKSelector.forward (gsa_ref.py:138-150): the k_eff
// largest of the row's valid scores (the reference maps -inf to -1e9, so
// valid scores always win and -inf picks come back with mask 0), plus the
// ascending index sort of gsa_opt.py:674-677.  Ties are broken toward the
// lower key index (torch.topk leaves tie order unspecified).
//
// One CTA (256 threads) per query row; n = min(q_pos0 + r + 1, Tkv) keys.
//  1. Stage the row as order-preserving uint32 keys (shared memory when the
//     row fits, else re-read from global/L2) and reduce min/max of the finite
//     keys and the finite count.
//  2. Radix select of the k-th largest key, MSB first with 11-bit digits,
//     starting at the highest bit in which the row's min and max keys differ
//     (scores of one row share their top exponent bits, so a fixed first
//     digit would put every key in one bin).  After the first digit the keys
//     of the threshold bin are compacted into a short candidate list and the
//     remaining digits scan only that list.
//  3. Emit: each warp owns a contiguous segment of the row and writes one
//     bitmask word per 32 keys straight from a ballot.  When column lists are
//     requested, or only part of the keys equal to the threshold are taken
//     (exact ties), a counting phase and a scan of the 8 warp totals first give
//     every warp its output offset and its share of the tied keys (lowest
//     index first); the bitmask-only forward path normally skips it.
#include "kernels.h"

namespace gsa {
namespace {

constexpr int kTopkThreads = 256;
constexpr int kTopkWarps = kTopkThreads / 32;
constexpr int kBins = 2048;          // 11-bit digits
constexpr int kDigitBits = 11;
constexpr int kCandCap = 1024;       // candidate list capacity
// Rows up to this many keys are staged in shared memory (128 KB).
constexpr int kTopkStageMax = 32768;

__device__ __forceinline__ uint32_t ord_key(float f) {
  const uint32_t x = __float_as_uint(f);
  return (x & 0x80000000u) ? ~x : (x | 0x80000000u);
}
// ord_key(-inf) (0xFF800000 inverted): below every finite key.
constexpr uint32_t kNegInfKey = 0x007FFFFFu;

struct TopkShared {
  int hist[kBins];
  uint32_t cand_key[kCandCap];
  int cand_idx[kCandCap];
  int warp_a[kTopkWarps];
  int warp_b[kTopkWarps];
  uint32_t red_min[kTopkWarps];
  uint32_t red_max[kTopkWarps];
  int red_cnt[kTopkWarps];
  int n_cand;
  int sh_digit, sh_above, sh_bin;
};

template <bool STAGED>
__global__ void __launch_bounds__(kTopkThreads) topk_kernel(
    const float* __restrict__ scores, int64_t score_stride, int Tq, int Tkv, int q_pos0, int k_sel,
    int32_t* __restrict__ indices, uint8_t* __restrict__ mask, uint32_t* __restrict__ bitmask,
    int64_t bm_words) {
  extern __shared__ uint32_t skeys[];
  __shared__ TopkShared sh;

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const uint32_t lt_mask = (1u << lane) - 1u;
  const int64_t row = blockIdx.x;  // b * Tq + r
  const int r = static_cast<int>(row % Tq);
  const int n = min(q_pos0 + r + 1, Tkv);
  const float* srow = scores + row * score_stride;
  int32_t* irow = indices ? indices + row * k_sel : nullptr;
  uint8_t* mrow = mask ? mask + row * k_sel : nullptr;
  uint32_t* brow = bitmask ? bitmask + row * bm_words : nullptr;

  auto key_at = [&](int j) -> uint32_t {
    if (STAGED) return skeys[j];
    return ord_key(__ldg(srow + j));
  };

  // ---- 1. stage + min/max/count of finite keys.  16-byte loads, four in
  // flight per thread, when the row is 16-byte aligned; scalar otherwise.
  uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
  int nfin = 0;
  auto note = [&](uint32_t u) {
    if (u != kNegInfKey) {
      kmin = min(kmin, u);
      kmax = max(kmax, u);
      ++nfin;
    }
  };
  auto take = [&](int j, float f) {
    const uint32_t u = ord_key(f);
    if (STAGED) skeys[j] = u;
    note(u);
  };
  int j_vec = 0;
  if ((reinterpret_cast<uintptr_t>(srow) & 15u) == 0) {
    const float4* s4 = reinterpret_cast<const float4*>(srow);
    const int nv = n >> 2;
    constexpr int U = 8;
    for (int v0 = 0; v0 < nv; v0 += U * kTopkThreads) {
      float4 f[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int v = v0 + u * kTopkThreads + tid;
        f[u] = v < nv ? __ldg(s4 + v) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int v = v0 + u * kTopkThreads + tid;
        if (v < nv) {
          const uint4 k4 = make_uint4(ord_key(f[u].x), ord_key(f[u].y), ord_key(f[u].z),
                                      ord_key(f[u].w));
          if (STAGED) reinterpret_cast<uint4*>(skeys)[v] = k4;  // one 16-byte store
          note(k4.x);
          note(k4.y);
          note(k4.z);
          note(k4.w);
        }
      }
    }
    j_vec = nv << 2;
  }
  for (int j = j_vec + tid; j < n; j += kTopkThreads) take(j, __ldg(srow + j));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    kmin = min(kmin, __shfl_xor_sync(0xFFFFFFFFu, kmin, o));
    kmax = max(kmax, __shfl_xor_sync(0xFFFFFFFFu, kmax, o));
    nfin += __shfl_xor_sync(0xFFFFFFFFu, nfin, o);
  }
  if (lane == 0) {
    sh.red_min[warp] = kmin;
    sh.red_max[warp] = kmax;
    sh.red_cnt[warp] = nfin;
  }
  __syncthreads();
  kmin = 0xFFFFFFFFu;
  kmax = 0u;
  nfin = 0;
#pragma unroll
  for (int w = 0; w < kTopkWarps; ++w) {
    kmin = min(kmin, sh.red_min[w]);
    kmax = max(kmax, sh.red_max[w]);
    nfin += sh.red_cnt[w];
  }

  // Selection = keys in a class above `prefix` (under `pmask`), plus the
  // first `krem` keys (by index) of the class equal to `prefix`.  `fin_only`
  // excludes -inf keys from both.
  uint32_t prefix = 0, pmask = 0;
  int krem = k_sel;
  bool fin_only = false;
  bool eq_all = true;  // every key of the equal class is taken (no tie to split)
  if (n <= k_sel) {
    // everything is taken (prefix/pmask = 0: one class, krem >= n)
  } else if (nfin <= k_sel) {
    // all finite keys, then the lowest-index -inf keys.  Those are listed with
    // mask 0 but never set a bitmask bit, so only column lists rank them
    // (need_rank below is then already forced by indices/mask).
    pmask = 0xFFFFFFFFu;
    prefix = kNegInfKey;
    krem = k_sel - nfin;
  } else {
    fin_only = true;
    const uint32_t diff = kmin ^ kmax;
    int hb = diff ? 31 - __clz(diff) : 0;      // highest differing bit
    pmask = hb >= 31 ? 0u : ~((2u << hb) - 1u);
    prefix = kmin & pmask;
    int shift = max(hb - (kDigitBits - 1), 0);
    bool use_cand = false;
    while (true) {
      const uint32_t dmask = (hb >= 31 ? 0xFFFFFFFFu : ((2u << hb) - 1u)) >> shift << shift;
      for (int b = tid; b < kBins; b += kTopkThreads) sh.hist[b] = 0;
      __syncthreads();
      if (!use_cand) {
        for (int j = tid; j < n; j += kTopkThreads) {
          const uint32_t u = key_at(j);
          if (u != kNegInfKey && (u & pmask) == prefix)
            atomicAdd(&sh.hist[(u & dmask) >> shift], 1);
        }
      } else {
        for (int c = tid; c < sh.n_cand; c += kTopkThreads) {
          const uint32_t u = sh.cand_key[c];
          if ((u & pmask) == prefix) atomicAdd(&sh.hist[(u & dmask) >> shift], 1);
        }
      }
      __syncthreads();
      // suffix scan: thread t owns bins kBpt*t .. kBpt*t+kBpt-1 counted from the top bin down
      constexpr int kBpt = kBins / kTopkThreads;
      int own[kBpt], loc = 0;
#pragma unroll
      for (int q = 0; q < kBpt; ++q) {
        own[q] = sh.hist[kBins - 1 - (kBpt * tid + q)];
        loc += own[q];
      }
      int inc = loc;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xFFFFFFFFu, inc, o);
        if (lane >= o) inc += y;
      }
      if (lane == 31) sh.warp_a[warp] = inc;
      __syncthreads();
      int before = inc - loc;
      for (int w = 0; w < warp; ++w) before += sh.warp_a[w];
      if (before < krem && before + loc >= krem) {
        int cum = before;
#pragma unroll
        for (int q = 0; q < kBpt; ++q) {
          if (cum < krem && cum + own[q] >= krem) {
            sh.sh_digit = kBins - 1 - (kBpt * tid + q);
            sh.sh_above = cum;
            sh.sh_bin = own[q];
          }
          cum += own[q];
        }
      }
      __syncthreads();
      const uint32_t digit = static_cast<uint32_t>(sh.sh_digit);
      krem -= sh.sh_above;
      const int bin_count = sh.sh_bin;
      prefix |= digit << shift;
      pmask |= dmask;
      if (bin_count == krem) break;                // the whole class is taken
      if (shift == 0) {                            // bits exhausted: exact ties
        eq_all = false;
        break;
      }
      // compact the class into the candidate list once it is short enough
      if (!use_cand && bin_count <= kCandCap) {
        if (tid == 0) sh.n_cand = 0;
        __syncthreads();
        for (int j = tid; j < n; j += kTopkThreads) {
          const uint32_t u = key_at(j);
          if (u != kNegInfKey && (u & pmask) == prefix) {
            const int c = atomicAdd(&sh.n_cand, 1);
            sh.cand_key[c] = u;
            sh.cand_idx[c] = j;
          }
        }
        use_cand = true;
      }
      __syncthreads();
      hb = shift - 1;
      shift = max(hb - (kDigitBits - 1), 0);
    }
    __syncthreads();
  }

  // ---- 3. emit in ascending index order (warp-contiguous segments)
  const int span = ((n + 31) / 32) * 32;
  const int seg = ((span / 32 + kTopkWarps - 1) / kTopkWarps) * 32;  // keys per warp
  const int s0 = min(warp * seg, span), s1 = min(s0 + seg, span);
  auto classify = [&](int j, bool& gt, bool& eq, bool& fin) {
    const bool valid = j < n;
    const uint32_t u = valid ? key_at(j) : kNegInfKey;
    fin = u != kNegInfKey;
    const bool fin_ok = !fin_only || fin;
    const uint32_t m = u & pmask;
    gt = valid && fin_ok && m > prefix;
    eq = valid && fin_ok && m == prefix;
  };
  const bool need_rank = irow != nullptr || mrow != nullptr || !eq_all;
  if (!need_rank) {
    // bitmask only, whole equal class taken: one pass, no counting
    for (int j0 = s0; j0 < s1; j0 += 32) {
      bool gt, eq, fin;
      classify(j0 + lane, gt, eq, fin);
      const uint32_t liveb = __ballot_sync(0xFFFFFFFFu, (gt || eq) && fin);
      if (lane == 0 && (j0 >> 5) < bm_words) brow[j0 >> 5] = liveb;
    }
  } else {
    int gt_w = 0, eq_w = 0;
    for (int j0 = s0; j0 < s1; j0 += 32) {
      bool gt, eq, fin;
      classify(j0 + lane, gt, eq, fin);
      gt_w += __popc(__ballot_sync(0xFFFFFFFFu, gt));
      eq_w += __popc(__ballot_sync(0xFFFFFFFFu, eq));
    }
    if (lane == 0) {
      sh.warp_a[warp] = gt_w;
      sh.warp_b[warp] = eq_w;
    }
    __syncthreads();
    int eq_before = 0, sel_before = 0;
    for (int w = 0; w < warp; ++w) {
      const int e = sh.warp_b[w];
      sel_before += sh.warp_a[w] + max(0, min(krem - eq_before, e));
      eq_before += e;
    }
    int eq_run = eq_before;
    int out = sel_before;
    for (int j0 = s0; j0 < s1; j0 += 32) {
      const int j = j0 + lane;
      bool gt, eq, fin;
      classify(j, gt, eq, fin);
      const uint32_t eqb = __ballot_sync(0xFFFFFFFFu, eq);
      const bool sel = gt || (eq && eq_run + __popc(eqb & lt_mask) < krem);
      eq_run += __popc(eqb);
      const uint32_t selb = __ballot_sync(0xFFFFFFFFu, sel);
      const bool live = sel && fin;
      if (sel) {
        const int pos = out + __popc(selb & lt_mask);
        if (irow) irow[pos] = j;
        if (mrow) mrow[pos] = live ? 1 : 0;
      }
      const uint32_t liveb = __ballot_sync(0xFFFFFFFFu, live);
      if (brow && lane == 0 && (j0 >> 5) < bm_words) brow[j0 >> 5] = liveb;
      out += __popc(selb);
    }
  }
  if (brow) {
    for (int64_t wd = span / 32 + tid; wd < bm_words; wd += kTopkThreads) brow[wd] = 0u;
  }
  // filler slots after the selected ones (n < k_sel): future positions, masked
  const int n_sel = min(n, k_sel);
  for (int s = n_sel + tid; s < k_sel; s += kTopkThreads) {
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
