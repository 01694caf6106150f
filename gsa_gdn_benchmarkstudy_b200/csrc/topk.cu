// topk.cu — per-row top-k selection over causal indexer scores.
//
// Replaces AdaptiveTopKSelector.forward (gsa_ref.py:138-150): the k_eff
// largest of the row's valid scores (the reference maps -inf to -1e9, so
// valid scores always win and -inf picks come back with mask 0), plus the
// ascending index sort of gsa_opt.py:674-677.  Ties are broken toward the
// lower key index (torch.topk leaves tie order unspecified).
//
// One CTA of 128 threads per query row; the row has n = min(q_pos0 + r + 1,
// Tkv) keys.  Scores become order-preserving uint32 keys (ord_key).
//
// Fast path (rows with n > k, the common case):
//  1. One key per thread, sampled evenly over the row, gives a key range
//     [lo, hi], widened by a quarter on each side; bin(u) = clamp((u - lo) >>
//     shift, 0, 2047) is monotonic in u.  When lo is the key of a
//     non-negative float (indexer scores always are), the same bins come from
//     the raw float bits with fewer integer ops (PosBins).
//  2. One read of the row builds the 2048-bin histogram of finite keys.
//  3. The bin holding the k-th largest key is found by a suffix scan.
//  4. A second read emits, per 32 keys, a ballot of the keys in higher bins
//     into a shared-memory copy of the row's bitmask and collects the keys of
//     the threshold bin into a candidate list.
//  5. Candidates are ranked exactly by (key desc, index asc); the top ones are
//     OR'd into the bitmask, which is then written out coalesced (and turned
//     into an ascending column list when one is requested).
// Rows the fast path cannot finish (n <= k, few finite scores, a degenerate
// sample range or an over-full threshold bin — e.g. heavy exact ties) take the
// exact path: an MSB-first 11-bit radix select starting at the highest bit in
// which the row's min and max keys differ, with candidate compaction, and a
// warp-segmented emit.  Both paths implement the same selection rule.
#include <algorithm>
#include <cstddef>
#include <type_traits>

#include "kernels.h"

namespace gsa {
namespace {

#ifndef GSA_TOPK_THREADS
#define GSA_TOPK_THREADS 128
#endif
constexpr int kTopkThreads = GSA_TOPK_THREADS;  // threads per row (a power of two, 128..1024)
static_assert(kTopkThreads >= 128 && kTopkThreads <= 1024 && (kTopkThreads & (kTopkThreads - 1)) == 0,
              "threads per row");
constexpr int kTopkWarps = kTopkThreads / 32;
constexpr int kBins = 2048;   // 11-bit digits / histogram bins
// 32-key groups per emit step, whose loads are in flight together.  Measured
// top-k times for 4 / 8 / 16 groups: at T=64K, where the emit pass reads the
// score rows back from DRAM, 3.66 / 3.34 / 3.09 ms; at T=16K, where they come
// from L2, 0.280 / 0.278 / 0.289 ms.  Key ranges of kLongKeyRange or more take
// the long step, shorter ones the short step (one kernel instance each).
constexpr int kEmitShort = 4;
constexpr int kEmitLong = 16;
constexpr int kLongKeyRange = 32768;
constexpr int kDigitBits = 11;
constexpr int kCandCap = 1024;  // candidate list capacity
constexpr int kMaxWords = 2048; // bitmask words held in shared memory (Tkv <= 65536)

// -0.0 maps to the key of +0.0: the two compare equal (as in torch.topk), so
// they tie and the lower column index wins.
__device__ __forceinline__ uint32_t ord_key(float f) {
  const uint32_t x0 = __float_as_uint(f);
  const uint32_t x = x0 == 0x80000000u ? 0u : x0;
  return (x & 0x80000000u) ? ~x : (x | 0x80000000u);
}
// ord_key(-inf) (0xFF800000 inverted): below every finite key.
constexpr uint32_t kNegInfKey = 0x007FFFFFu;

// Bin maps of the fast path.  Both give bin(f) = clamp((ord_key(f) - lo) >>
// shift, 0, 2047) for finite f (-1 for -inf), monotonic in the key order, and
// after set_threshold(b) classify f as gt (bin > b) / eq (bin == b).
struct OrdBins {
  static constexpr bool kRawBits = false;
  uint32_t lo;
  int shift;
  int bstar = 0;
  __device__ OrdBins(uint32_t lo_, int shift_) : lo(lo_), shift(shift_) {}
  __device__ __forceinline__ int bin(float f) const {
    const uint32_t u = ord_key(f);
    if (u == kNegInfKey) return -1;
    return u <= lo ? 0 : min(static_cast<int>((u - lo) >> shift), kBins - 1);
  }
  // histogram slot of f and 1 if f counts (finite), without a branch
  __device__ __forceinline__ int hist_bin(float f, int& inc) const {
    const uint32_t u = ord_key(f);
    inc = u != kNegInfKey ? 1 : 0;
    return u <= lo ? 0 : min(static_cast<int>((u - lo) >> shift), kBins - 1);
  }
  __device__ __forceinline__ void set_threshold(int b) { bstar = b; }
  __device__ __forceinline__ void classify(float f, bool& gt, bool& eq) const {
    const int bn = bin(f);
    gt = bn > bstar;
    eq = bn == bstar;
  }
};

// The same map when lo is the key of a non-negative float, with raw = its
// bits (lo - 0x80000000): non-negative floats' bits are already in key
// order, every negative float (and -0.0) falls in bin 0 either way, so
// bin(f) = clamp((max(bits, 0) - raw) >> shift, 0, 2047) as signed ints and
// the gt / eq tests become two compares against the threshold bin's edges.
// kFinite: the caller guarantees no -inf among the row's keys (the fused
// indexer + top-k call: the indexer writes finite scores), so every key counts.
template <bool kFinite>
struct PosBins {
  static constexpr bool kRawBits = true;
  int raw;
  int shift;
  int lo_edge = 0, hi_m1 = 0;
  static constexpr int kNegInfBits = static_cast<int>(0xFF800000u);
  __device__ PosBins(uint32_t raw_, int shift_) : raw(static_cast<int>(raw_)), shift(shift_) {}
  // -inf is a negative float: bin 0, not counted.  max(x, raw) - raw is
  // max(max(x, 0) - raw, 0) for raw >= 0.
  __device__ __forceinline__ int hist_bin(float f, int& inc) const {
    const int x = __float_as_int(f);
    inc = (kFinite || x != kNegInfBits) ? 1 : 0;
    return min((max(x, raw) - raw) >> shift, kBins - 1);
  }
  // bin(f) > b  <=>  bits > hi_m1;  bin(f) >= b  <=>  bits >= lo_edge (b > 0).
  // A key of bin b exists (b holds the k-th largest), so lo_edge fits in int.
  __device__ __forceinline__ void set_threshold(int b) {
    const long long lo64 = static_cast<long long>(raw) + (static_cast<long long>(b) << shift);
    const long long hi64 = static_cast<long long>(raw) + (static_cast<long long>(b + 1) << shift) - 1;
    lo_edge = b == 0 ? INT_MIN : static_cast<int>(min(lo64, static_cast<long long>(INT_MAX)));
    hi_m1 = (b == kBins - 1 || hi64 > INT_MAX) ? INT_MAX : static_cast<int>(hi64);
  }
  __device__ __forceinline__ void classify(float f, bool& gt, bool& eq) const {
    const int x = __float_as_int(f);
    gt = x > hi_m1;
    eq = !gt && x >= lo_edge && x != kNegInfBits;
  }
};

// Per-instance shared-memory sizes.  The short-range instance (key range <
// kLongKeyRange, rows of at most kLongKeyRange / 32 bitmask words) keeps 512
// candidates: its smaller footprint (16.5 against 24.7 KB) leaves more of the
// SM's L1 to the rows' second read at the same 8 CTAs per SM (registers
// bound those).  Measured at T=16K: top-k 0.255 -> 0.235 ms, indexer + top-k
// 0.472 -> 0.441 ms; a lower register cap for more CTAs per SM (10, 11 or 12)
// and a larger L1 carve-out at fewer CTAs were slower.  The long instance
// keeps kCandCap.
constexpr int kShortCandCap = 512;
template <int kGroups>
constexpr int topk_words() { return kGroups == kEmitLong ? kMaxWords : kLongKeyRange / 32; }
template <int kGroups>
constexpr int topk_cand_cap() { return kGroups == kEmitLong ? kCandCap : kShortCandCap; }

template <int kWords, int kCap>
struct alignas(16) TopkShared {
  static constexpr int kNumWords = kWords;
  static constexpr int kNumCand = kCap;
  int hist[kBins];
  uint32_t cand_key[kCap];
  int cand_idx[kCap];
  uint32_t bits[kWords];
  int warp_a[kTopkWarps];
  int warp_b[kTopkWarps];
  uint32_t red_min[kTopkWarps];
  uint32_t red_max[kTopkWarps];
  int red_cnt[kTopkWarps];
  int n_cand;
  int sh_digit, sh_above, sh_bin;
};

// Block-wide reduction of (min, max, sum) into every thread.
template <typename Sh>
__device__ __forceinline__ void block_minmax_count(Sh& sh, uint32_t& kmin, uint32_t& kmax,
                                                   int& cnt) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    kmin = min(kmin, __shfl_xor_sync(0xFFFFFFFFu, kmin, o));
    kmax = max(kmax, __shfl_xor_sync(0xFFFFFFFFu, kmax, o));
    cnt += __shfl_xor_sync(0xFFFFFFFFu, cnt, o);
  }
  if (lane == 0) {
    sh.red_min[warp] = kmin;
    sh.red_max[warp] = kmax;
    sh.red_cnt[warp] = cnt;
  }
  __syncthreads();
  kmin = 0xFFFFFFFFu;
  kmax = 0u;
  cnt = 0;
#pragma unroll
  for (int w = 0; w < kTopkWarps; ++w) {
    kmin = min(kmin, sh.red_min[w]);
    kmax = max(kmax, sh.red_max[w]);
    cnt += sh.red_cnt[w];
  }
  __syncthreads();
}

// Suffix scan over sh.hist (bins counted from the top down): finds the bin
// holding the krem-th largest key; sets sh_digit / sh_above / sh_bin (left
// unset when the histogram holds fewer than krem keys).  Returns the
// histogram's total count, in every thread.
template <int kNB = kBins, typename Sh>
__device__ __forceinline__ int find_threshold_bin(Sh& sh, int krem) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int kBpt = kNB / kTopkThreads;
  static_assert(kBpt % 4 == 0 && offsetof(Sh, hist) % 16 == 0, "16-byte histogram reads");
  // this thread's bins kNB-1-kBpt*tid down to kNB-kBpt*(tid+1): one contiguous
  // block, read as 16-byte vectors (scalar reads at a stride of kBpt words
  // would conflict kBpt/2-fold across the warp)
  int own[kBpt], loc = 0;
  {
    const int4* blk = reinterpret_cast<const int4*>(sh.hist + kNB - kBpt * (tid + 1));
#pragma unroll
    for (int v = 0; v < kBpt / 4; ++v) {
      const int4 x = blk[v];
      own[kBpt - 1 - 4 * v] = x.x;
      own[kBpt - 2 - 4 * v] = x.y;
      own[kBpt - 3 - 4 * v] = x.z;
      own[kBpt - 4 - 4 * v] = x.w;
    }
#pragma unroll
    for (int q = 0; q < kBpt; ++q) loc += own[q];
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
  int total = 0;
#pragma unroll
  for (int w = 0; w < kTopkWarps; ++w) total += sh.warp_a[w];
  if (before < krem && before + loc >= krem) {
    int cum = before;
#pragma unroll
    for (int q = 0; q < kBpt; ++q) {
      if (cum < krem && cum + own[q] >= krem) {
        sh.sh_digit = kNB - 1 - (kBpt * tid + q);
        sh.sh_above = cum;
        sh.sh_bin = own[q];
      }
      cum += own[q];
    }
  }
  __syncthreads();
  return total;
}

// Ascending column list (irow) and mask 1 (mrow) of the set bits of
// sh.bits[0, nwords), in order; every set bit is a finite pick.
template <typename Sh>
__device__ __forceinline__ void bits_to_lists(Sh& sh, int nwords, int32_t* irow,
                                              uint8_t* mrow) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int wseg = (nwords + kTopkWarps - 1) / kTopkWarps;
  const int w0 = min(warp * wseg, nwords), w1 = min(w0 + wseg, nwords);
  int cnt = 0;
  for (int w = w0 + lane; w < w1; w += 32) cnt += __popc(sh.bits[w]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xFFFFFFFFu, cnt, o);
  if (lane == 0) sh.warp_a[warp] = cnt;
  __syncthreads();
  int out = 0;
  for (int w = 0; w < warp; ++w) out += sh.warp_a[w];
  for (int wb = w0; wb < w1; wb += 32) {
    const int w = wb + lane;
    const uint32_t word = w < w1 ? sh.bits[w] : 0u;
    const int pc = __popc(word);
    int incl = pc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
    int pos = out + incl - pc;
    uint32_t rest = word;
    while (rest) {
      const int bit = __ffs(rest) - 1;
      rest &= rest - 1;
      if (irow) irow[pos] = w * 32 + bit;
      if (mrow) mrow[pos] = 1;
      ++pos;
    }
    out += __shfl_sync(0xFFFFFFFFu, incl, 31);
  }
}

// k of one row in adaptive mode (gsa_explained.ipynb, "Adaptive Top-K" cell):
//   avg_var = mean over the batch's rows of row_var, clamped to >= 1e-6
//   k = clamp(floor(k_base * avg_var / max(row_var, 1e-6)), k_min, k_max)
// The mean is the double-precision sum of the row variances over the row
// count, rounded once to fp32 (torch's fp32 mean can differ from it in the
// last ulp, and then a row whose ratio lies that close to an integer gets a k
// one apart); the rest is fp32 with round-to-nearest multiply and divide, as
// torch computes it.  A NaN row variance gives k_max.
__device__ __forceinline__ int adaptive_row_k(const AdaptiveK& ad, int64_t row) {
  const float avg =
      fmaxf(static_cast<float>(*ad.var_sum / static_cast<double>(ad.var_rows)), 1e-6f);
  const float t = __fdiv_rn(__fmul_rn(static_cast<float>(ad.k_base), avg),
                            fmaxf(ad.row_var[row], 1e-6f));
  float kf = floorf(t);
  kf = fmaxf(kf, static_cast<float>(ad.k_min));
  kf = fminf(kf, static_cast<float>(ad.k_max));
  return static_cast<int>(kf);
}

// Selection of one row (the whole CTA): the k_sel best of the row's n valid
// scores srow[0, n) into irow / mrow (k_width slots; NULL = not wanted) and
// brow (bm_words words; NULL = not wanted).
template <bool kFinite, int kGroups, typename Sh>
__device__ __forceinline__ void topk_row(Sh& sh, const float* __restrict__ srow, int n,
                                         int Tkv, int k_sel, int k_width, int32_t* irow,
                                         uint8_t* mrow, uint32_t* brow, int64_t bm_words) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const uint32_t lt_mask = (1u << lane) - 1u;
  const bool vec_ok = (reinterpret_cast<uintptr_t>(srow) & 15u) == 0;
  const int nwords = (n + 31) / 32;

  auto key_at = [&](int j) -> uint32_t { return ord_key(__ldg(srow + j)); };

  if (k_sel <= 0) {  // nothing selected: an all-zero bitmask and masked slots
    if (brow)
      for (int64_t w = tid; w < bm_words; w += kTopkThreads) brow[w] = 0u;
    for (int s = tid; s < k_width; s += kTopkThreads) {
      if (irow) irow[s] = min(s, Tkv - 1);
      if (mrow) mrow[s] = 0;
    }
    return;
  }
  if (kFinite && n <= k_sel) {
    // every key of the row is selected (finite rows: no -inf to leave out), so
    // the selection is columns [0, n) without reading a score
    if (brow) {
      const int full = n >> 5, rem = n & 31;
      for (int64_t w = tid; w < bm_words; w += kTopkThreads)
        brow[w] = w < full ? 0xFFFFFFFFu : (w == full && rem ? (1u << rem) - 1u : 0u);
    }
    for (int s = tid; s < k_width; s += kTopkThreads) {
      if (irow) irow[s] = min(s, Tkv - 1);  // s itself below n; filler above
      if (mrow) mrow[s] = s < n ? 1 : 0;
    }
    return;
  }

  // =================================================================== fast path
  bool done = false;
  if (n > k_sel && nwords <= Sh::kNumWords) {
    // float4 loads per thread in flight in the histogram pass: 8 when the rows
    // come from L2 (key range under 32K: 0.276 -> 0.268 ms at T=16K), 4 when
    // they come from DRAM (8 cost 12% at T=64K).  Rows without -inf (kFinite)
    // issue the first batch here, beside the sample loads, so that its latency
    // overlaps the range reduction (T=16K: indexer + top-k 0.417 -> 0.413 ms,
    // T=8K x 8: 0.891 -> 0.877 ms); elsewhere the batch held across the
    // reduction cost registers (56 -> 72) and time.
    constexpr int U = kGroups == kEmitLong ? 4 : 8;
    const float4* s4 = reinterpret_cast<const float4*>(srow);
    const int nv = vec_ok ? n >> 2 : 0;
    float4 f0[U];
    if constexpr (kFinite) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int v = u * kTopkThreads + tid;
        f0[u] = v < nv ? __ldg(s4 + v) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    // 1. sample range
    uint32_t smin = 0xFFFFFFFFu, smax = 0u;
    int sfin = 0;
    {
      // tid * (n - 1) < 2^31 here (n <= 32 * kMaxWords)
      const int p = static_cast<int>(static_cast<uint32_t>(tid) * static_cast<uint32_t>(n - 1) /
                                     static_cast<uint32_t>(kTopkThreads - 1));
      const uint32_t u = key_at(p);
      if (u != kNegInfKey) {
        smin = u;
        smax = u;
        sfin = 1;
      }
    }
    for (int b = tid; b < kBins / 4; b += kTopkThreads)
      reinterpret_cast<int4*>(sh.hist)[b] = make_int4(0, 0, 0, 0);
    for (int w = tid; w < nwords; w += kTopkThreads) sh.bits[w] = 0u;
    if (tid == 0) sh.n_cand = 0;
    block_minmax_count(sh, smin, smax, sfin);
    if (sfin > 0 && smax > smin) {
      const uint32_t width = smax - smin;
      const uint32_t margin = width >> 2;
      const uint32_t lo = smin > margin ? smin - margin : 0u;
      const uint32_t span_w = min(0xFFFFFFFFu - lo, width + 2 * margin);
      const int shift = max(0, 32 - __clz(span_w) - kDigitBits);
      // Steps 2-5 for one bin map (OrdBins, or PosBins when the range starts
      // at a non-negative float: the same bins from fewer integer ops).
      // Returns false (block-uniformly) when the row needs the exact path.
      auto fast = [&](auto bins) -> bool {
        // 2. histogram of finite keys
        auto hist_key = [&](float f) {
          int inc;
          const int bn = bins.hist_bin(f, inc);
          atomicAdd(&sh.hist[bn], inc);
        };
        auto hist_batch = [&](const float4 (&f)[U], int v0) {
#pragma unroll
          for (int u = 0; u < U; ++u) {
            if (v0 + u * kTopkThreads + tid < nv) {
              hist_key(f[u].x);
              hist_key(f[u].y);
              hist_key(f[u].z);
              hist_key(f[u].w);
            }
          }
        };
        int v_first = 0;
        if constexpr (kFinite) {
          hist_batch(f0, 0);
          v_first = U * kTopkThreads;
        }
        for (int v0 = v_first; v0 < nv; v0 += U * kTopkThreads) {
          float4 f[U];
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int v = v0 + u * kTopkThreads + tid;
            f[u] = v < nv ? __ldg(s4 + v) : make_float4(0.f, 0.f, 0.f, 0.f);
          }
          hist_batch(f, v0);
        }
        const int jv = nv << 2;
        for (int j = jv + tid; j < n; j += kTopkThreads) hist_key(__ldg(srow + j));
        __syncthreads();
        // finite keys = histogram total
        // 3. threshold bin; the scan also counts the finite keys
        const int nfin = find_threshold_bin(sh, k_sel);
        if (nfin <= k_sel) return false;
        const int bstar = sh.sh_digit;
        const int krem = k_sel - sh.sh_above;
        const int bcount = sh.sh_bin;
        if (bcount > Sh::kNumCand) return false;
        bins.set_threshold(bstar);
        // 4. bits for higher bins, candidates of the threshold bin; G 32-key groups per
        // step, whose loads are in flight together
        constexpr int G = kGroups;
        // keys per warp: a multiple of one step, so a step's words go out as
        // 16-byte stores
        const int seg = ((nwords + G * kTopkWarps - 1) / (G * kTopkWarps)) * (G * 32);
        const int s0 = min(warp * seg, nwords * 32), s1 = min(s0 + seg, nwords * 32);
        const float kNegInf = -__int_as_float(0x7F800000);
        auto emit_group = [&](int j0, float f) {
          bool gt, eq;
          bins.classify(f, gt, eq);
          const uint32_t hib = __ballot_sync(0xFFFFFFFFu, gt);
          const uint32_t eqb = __ballot_sync(0xFFFFFFFFu, eq);
          if (eqb) {  // warp-uniform; one atomic per warp
            int base = 0;
            if (lane == 0) base = atomicAdd(&sh.n_cand, __popc(eqb));
            base = __shfl_sync(0xFFFFFFFFu, base, 0);
            if (eq) {
              const int c = base + __popc(eqb & lt_mask);
              sh.cand_key[c] = ord_key(f);
              sh.cand_idx[c] = j0 + lane;
            }
          }
          if (lane == 0) sh.bits[j0 >> 5] = hib;
        };
        using BT = typename std::decay<decltype(bins)>::type;
        int full_end;
        if constexpr (BT::kRawBits) {
          // whole steps inside the row: one compare per key for the bits, and the
          // threshold-bin keys (a few per row) collected only in steps that have one
          const int hi_m1 = bins.hi_m1, lo_edge = bins.lo_edge;
          full_end = s0 + max(0, min(s1, n) - s0) / (G * 32) * (G * 32);
          // Short steps issue the next step's loads before this step's ballots
          // (T=16K: top-k 0.223 -> 0.214 ms; two steps ahead measured the same).
          // Long steps load in place: their 16 groups already keep the loads
          // in flight, and a second set would cost registers (64 -> 79).
          constexpr bool kPrefetch = G != kEmitLong;
          int xn[G];
          if (kPrefetch && s0 < full_end) {
#pragma unroll
            for (int g = 0; g < G; ++g) xn[g] = __float_as_int(__ldg(srow + s0 + lane + g * 32));
          }
          for (int jb = s0; jb < full_end; jb += G * 32) {
            int x[G];
            if constexpr (kPrefetch) {
#pragma unroll
              for (int g = 0; g < G; ++g) x[g] = xn[g];
              if (jb + G * 32 < full_end) {
#pragma unroll
                for (int g = 0; g < G; ++g)
                  xn[g] = __float_as_int(__ldg(srow + jb + G * 32 + lane + g * 32));
              }
            } else {
#pragma unroll
              for (int g = 0; g < G; ++g) x[g] = __float_as_int(__ldg(srow + jb + lane + g * 32));
            }
            uint32_t w[G];
            bool in = false;
#pragma unroll
            for (int g = 0; g < G; ++g) {
              w[g] = __ballot_sync(0xFFFFFFFFu, x[g] > hi_m1);
              in |= x[g] >= lo_edge && x[g] <= hi_m1;
            }
            if (lane == 0) {
#pragma unroll
              for (int q4 = 0; q4 < G / 4; ++q4)
                *reinterpret_cast<uint4*>(&sh.bits[(jb >> 5) + 4 * q4]) =
                    make_uint4(w[4 * q4], w[4 * q4 + 1], w[4 * q4 + 2], w[4 * q4 + 3]);
            }
            if (__any_sync(0xFFFFFFFFu, in)) {
#pragma unroll
              for (int g = 0; g < G; ++g) {
                const bool eq = x[g] >= lo_edge && x[g] <= hi_m1 && x[g] != BT::kNegInfBits;
                const uint32_t eqb = __ballot_sync(0xFFFFFFFFu, eq);
                if (eqb) {
                  int base = 0;
                  if (lane == 0) base = atomicAdd(&sh.n_cand, __popc(eqb));
                  base = __shfl_sync(0xFFFFFFFFu, base, 0);
                  if (eq) {
                    const int c = base + __popc(eqb & lt_mask);
                    sh.cand_key[c] = ord_key(__int_as_float(x[g]));
                    sh.cand_idx[c] = jb + g * 32 + lane;
                  }
                }
              }
            }
          }
        } else {
          full_end = s0 + max(0, min(s1, n) - s0) / (G * 32) * (G * 32);
          for (int jb = s0; jb < full_end; jb += G * 32) {  // whole steps inside the row
            float fg[G];
#pragma unroll
            for (int g = 0; g < G; ++g) fg[g] = __ldg(srow + jb + g * 32 + lane);
#pragma unroll
            for (int g = 0; g < G; ++g) emit_group(jb + g * 32, fg[g]);
          }
        }
        for (int j0 = full_end; j0 < s1; j0 += 32) {  // ragged tail, checked
          const int j = j0 + lane;
          emit_group(j0, j < n ? __ldg(srow + j) : kNegInf);
        }
        __syncthreads();
        // 5. exact rank among the candidates: (key desc, index asc)
        const int nc = sh.n_cand;
        for (int c = tid; c < nc; c += kTopkThreads) {
          const uint32_t u = sh.cand_key[c];
          const int ji = sh.cand_idx[c];
          // four candidates' loads in flight per step, compares without branches
          // (T=16K: indexer + top-k 0.413 -> 0.407 ms)
          int rank = 0;
          int o = 0;
          for (; o + 4 <= nc; o += 4) {
            uint32_t uo[4];
            int io[4];
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
              uo[q4] = sh.cand_key[o + q4];
              io[q4] = sh.cand_idx[o + q4];
            }
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4)
              rank += ((uo[q4] > u) | ((uo[q4] == u) & (io[q4] < ji))) ? 1 : 0;
          }
          for (; o < nc; ++o) {
            const uint32_t uo = sh.cand_key[o];
            const int io = sh.cand_idx[o];
            rank += ((uo > u) | ((uo == u) & (io < ji))) ? 1 : 0;
          }
          if (rank < krem) atomicOr(&sh.bits[ji >> 5], 1u << (ji & 31));
        }
        __syncthreads();
        if (brow) {
          for (int64_t w = tid; w < bm_words; w += kTopkThreads)
            brow[w] = w < nwords ? sh.bits[w] : 0u;
        }
        if (irow || mrow) bits_to_lists(sh, nwords, irow, mrow);
        return true;
      };
      done = lo >= 0x80000000u ? fast(PosBins<kFinite>(lo - 0x80000000u, shift))
                               : fast(OrdBins(lo, shift));
    }
    __syncthreads();
  }
  if (done) {
    // adaptive rows narrower than the output (k_sel < k_width): masked filler
    for (int s = k_sel + tid; s < k_width; s += kTopkThreads) {
      if (irow) irow[s] = min(s, Tkv - 1);
      if (mrow) mrow[s] = 0;
    }
    return;
  }

  // =================================================================== exact path
  uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
  int nfin = 0;
  for (int j = tid; j < n; j += kTopkThreads) {
    const uint32_t u = key_at(j);
    if (u != kNegInfKey) {
      kmin = min(kmin, u);
      kmax = max(kmax, u);
      ++nfin;
    }
  }
  block_minmax_count(sh, kmin, kmax, nfin);

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
    int hb = diff ? 31 - __clz(diff) : 0;  // highest differing bit
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
      find_threshold_bin(sh, krem);
      const uint32_t digit = static_cast<uint32_t>(sh.sh_digit);
      krem -= sh.sh_above;
      const int bin_count = sh.sh_bin;
      prefix |= digit << shift;
      pmask |= dmask;
      if (bin_count == krem) break;  // the whole class is taken
      if (shift == 0) {              // bits exhausted: exact ties
        eq_all = false;
        break;
      }
      // compact the class into the candidate list once it is short enough
      if (!use_cand && bin_count <= Sh::kNumCand) {
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

  // ---- emit in ascending index order (warp-contiguous segments)
  const int span = nwords * 32;
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
      if (brow && lane == 0 && (j0 >> 5) < bm_words) brow[j0 >> 5] = liveb;
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
  // filler slots after the selected ones (n < k_width): future positions, masked
  const int n_sel = min(n, k_sel);
  for (int s = n_sel + tid; s < k_width; s += kTopkThreads) {
    if (irow) irow[s] = min(s, Tkv - 1);
    if (mrow) mrow[s] = 0;
  }
}

template <bool kFinite, int kGroups>
__global__ void __launch_bounds__(kTopkThreads) topk_kernel(
    const float* __restrict__ scores, int64_t score_stride, int Tq, int Tkv, int q_pos0,
    int k_fixed, int k_width, AdaptiveK ad, int32_t* __restrict__ indices,
    uint8_t* __restrict__ mask, uint32_t* __restrict__ bitmask, int64_t bm_words) {
  __shared__ TopkShared<topk_words<kGroups>(), topk_cand_cap<kGroups>()> sh;
  const int64_t row = blockIdx.x;  // b * Tq + r
  const int r = static_cast<int>(row % Tq);
  const int n = min(q_pos0 + r + 1, Tkv);
  const int k_sel = ad.row_var ? adaptive_row_k(ad, row) : k_fixed;
  if (ad.row_k && threadIdx.x == 0) ad.row_k[row] = k_sel;
  topk_row<kFinite, kGroups>(sh, scores + row * score_stride, n, Tkv, k_sel, k_width,
                             indices ? indices + row * k_width : nullptr,
                             mask ? mask + row * k_width : nullptr,
                             bitmask ? bitmask + row * bm_words : nullptr, bm_words);
}

// ------------------------------------------------------------ row variance
// Adaptive mode's statistics (gsa_explained.ipynb, "Adaptive Top-K" cell):
// over the row's valid (finite-or-NaN, i.e. != -inf) scores,
//   mean = sum / max(count, 1),  var = sum((s - mean)^2) / max(count, 1).
// Two passes over the row (the second mostly from L2), block sums in a fixed
// order.

constexpr int kVarThreads = 256;
constexpr int kSumThreads = 1024;

__device__ __forceinline__ float block_sum_f(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kVarThreads / 32; ++w) t += red[w];
  __syncthreads();
  return t;
}

__global__ void __launch_bounds__(kVarThreads) row_variance_kernel(
    const float* __restrict__ scores, int64_t score_stride, int Tq, int Tkv, int q_pos0,
    float* __restrict__ row_var) {
  __shared__ float red[kVarThreads / 32];
  const int tid = threadIdx.x;
  const int64_t row = blockIdx.x;
  const int r = static_cast<int>(row % Tq);
  const int n = min(q_pos0 + r + 1, Tkv);
  const float* srow = scores + row * score_stride;
  const bool vec_ok = (reinterpret_cast<uintptr_t>(srow) & 15u) == 0;
  const int nv = vec_ok ? (n >> 2) : 0;
  const float4* s4 = reinterpret_cast<const float4*>(srow);
  const float kNegInf = -__int_as_float(0x7F800000);

  float sum = 0.f, cnt = 0.f;
  auto acc1 = [&](float f) {
    if (f != kNegInf) {
      sum += f;
      cnt += 1.f;
    }
  };
  for (int v = tid; v < nv; v += kVarThreads) {
    const float4 f = __ldg(s4 + v);
    acc1(f.x);
    acc1(f.y);
    acc1(f.z);
    acc1(f.w);
  }
  for (int j = 4 * nv + tid; j < n; j += kVarThreads) acc1(__ldg(srow + j));
  sum = block_sum_f(sum, red);
  cnt = block_sum_f(cnt, red);
  const float c = fmaxf(cnt, 1.f);
  const float mean = __fdiv_rn(sum, c);

  float m2 = 0.f;
  auto acc2 = [&](float f) {
    if (f != kNegInf) {
      const float d = f - mean;
      m2 = fmaf(d, d, m2);
    }
  };
  for (int v = tid; v < nv; v += kVarThreads) {
    const float4 f = __ldg(s4 + v);
    acc2(f.x);
    acc2(f.y);
    acc2(f.z);
    acc2(f.w);
  }
  for (int j = 4 * nv + tid; j < n; j += kVarThreads) acc2(__ldg(srow + j));
  m2 = block_sum_f(m2, red);
  if (tid == 0) row_var[row] = __fdiv_rn(m2, c);
}

// One CTA: sum of row_var[0, rows) in double, each thread a strided slice,
// then a fixed tree.
__global__ void __launch_bounds__(kSumThreads) var_sum_kernel(const float* __restrict__ row_var,
                                                              int64_t rows,
                                                              double* __restrict__ var_sum) {
  __shared__ double part[kSumThreads];
  double a = 0.0;
  for (int64_t i = threadIdx.x; i < rows; i += kSumThreads) a += static_cast<double>(row_var[i]);
  part[threadIdx.x] = a;
  __syncthreads();
  for (int h = kSumThreads / 2; h > 0; h >>= 1) {
    if (static_cast<int>(threadIdx.x) < h) part[threadIdx.x] += part[threadIdx.x + h];
    __syncthreads();
  }
  if (threadIdx.x == 0) *var_sum = part[0];
}

// ------------------------------------------------------------ fused selection
// The selection of gsa_indexer_topk on the tensor-core path (indexer_tk.cu):
//  1. the indexer scores each row against every key_step-th key (kSample);
//  2. select_threshold_kernel estimates each row's k-th score from its samples
//     and brackets it: hi at a sample rank z standard deviations above the
//     expected rank of the k-th key, lo z standard deviations below;
//  3. the indexer's kSelect pass turns keys above hi into bitmask bits and
//     keys in [lo, hi] into candidate lists, scores stored nowhere else;
//  4. rows whose bracket missed (or whose lists overflowed) get their full
//     score rows (kStoreFailed);
//  5. select_fixup_kernel completes each row exactly: the best (k - sure) of
//     its candidates by (score desc, key asc), or the plain top-k of a failed
//     row's full scores.  Either way the selection equals the top-k of the
//     same scores.
constexpr int kFixCap = kSelCandCap;  // candidates a row may hold
constexpr int kThrRows = kTopkWarps;  // threshold kernel: one warp per row
constexpr int kThrBins = 256;

// The float whose order-preserving key (ord_key) is u.
__device__ __forceinline__ float ord_to_float(uint32_t u) {
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u);
}

// Bin (of kThrBins, counted from the top by one warp) holding the rank-th
// largest sample, and the samples in higher bins.
__device__ __forceinline__ int warp_rank_bin(const int* hist, int rank, int& above) {
  const int lane = threadIdx.x & 31;
  int loc[kThrBins / 32], tot = 0;
#pragma unroll
  for (int q = 0; q < kThrBins / 32; ++q) {
    loc[q] = hist[kThrBins - 1 - (kThrBins / 32) * lane - q];
    tot += loc[q];
  }
  int incl = tot;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  int cum = incl - tot, bin = -1, ab = 0;
#pragma unroll
  for (int q = 0; q < kThrBins / 32; ++q) {
    if (cum < rank && cum + loc[q] >= rank) {
      bin = kThrBins - 1 - (kThrBins / 32) * lane - q;
      ab = cum;
    }
    cum += loc[q];
  }
  const uint32_t who = __ballot_sync(0xFFFFFFFFu, bin >= 0);
  const int src = who ? __ffs(who) - 1 : 0;
  above = __shfl_sync(0xFFFFFFFFu, ab, src);
  return __shfl_sync(0xFFFFFFFFu, bin, src);
}

__global__ void __launch_bounds__(kTopkThreads) select_threshold_kernel(
    const float* __restrict__ samples, int64_t stride, int64_t rows, int Tq, int Tkv, int q_pos0,
    int key_step, int key_off, int k_sel, float z, SelectRowStats* __restrict__ stats) {
  __shared__ int hist_all[kThrRows][kThrBins];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kThrRows + warp;
  if (row >= rows) return;  // warp-uniform; no block-wide barrier below
  int* hist = hist_all[warp];
  const int pos = q_pos0 + static_cast<int>(row % Tq);
  const int n = min(pos + 1, Tkv);
  const float kInf = __int_as_float(0x7F800000);
  float hi = -kInf, lo = -kInf;  // n <= k: every key is taken (all above hi)
  if (n > k_sel) {
    const int n_samples = Tkv > key_off ? (Tkv - key_off + key_step - 1) / key_step : 0;
    const int m = pos < key_off ? 0 : min((pos - key_off) / key_step + 1, n_samples);
    hi = kInf;  // without samples every key is a candidate
    if (m > 0) {
      // the number of samples above the k-th key follows a hypergeometric law:
      // mean m*p, variance m*p*(1-p)*(n-m)/(n-1), p = k/n
      const float p = static_cast<float>(k_sel) / static_cast<float>(n);
      const float mu = p * static_cast<float>(m);
      const float var = static_cast<float>(m) * p * (1.f - p) *
                        static_cast<float>(max(n - m, 0)) / static_cast<float>(max(n - 1, 1));
      const float sd = sqrtf(var);
      const int rho_hi = static_cast<int>(floorf(mu - z * sd)) - 1;  // ranks from the top, 1-based
      const int rho_lo = static_cast<int>(ceilf(mu + z * sd)) + 1;
      const float* srow = samples + row * stride;
      uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
      for (int i = lane; i < m; i += 32) {
        const uint32_t u = ord_key(srow[i]);
        kmin = min(kmin, u);
        kmax = max(kmax, u);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        kmin = min(kmin, __shfl_xor_sync(0xFFFFFFFFu, kmin, o));
        kmax = max(kmax, __shfl_xor_sync(0xFFFFFFFFu, kmax, o));
      }
      for (int bn = lane; bn < kThrBins; bn += 32) hist[bn] = 0;
      __syncwarp();
      const uint32_t width = kmax - kmin;
      const int shift = max(0, 32 - __clz(max(width, 1u)) - 8);  // (width >> shift) < 256
      for (int i = lane; i < m; i += 32) atomicAdd(&hist[(ord_key(srow[i]) - kmin) >> shift], 1);
      __syncwarp();
      int above = 0;
      if (rho_hi >= 1) {  // hi: top edge of the bin holding sample rank rho_hi
        const int bn = warp_rank_bin(hist, rho_hi, above);
        const uint64_t e = static_cast<uint64_t>(kmin) + (static_cast<uint64_t>(bn + 1) << shift) - 1u;
        hi = ord_to_float(static_cast<uint32_t>(min(e, static_cast<uint64_t>(kmax))));
      }
      if (rho_lo <= m) {  // lo: bottom edge of the bin holding sample rank rho_lo
        const int bn = warp_rank_bin(hist, rho_lo, above);
        lo = ord_to_float(kmin + (static_cast<uint32_t>(bn) << shift));
      }
    }
  }
  if (lane == 0) {
    SelectRowStats st;
    st.hi = hi;
    st.lo = lo;
    st.sure = 0;
    st.ncand = 0;
    st.flags = 0;
    st.pad[0] = st.pad[1] = st.pad[2] = 0;
    stats[row] = st;
  }
}

// One thread per row: marks the indexer tile (tile_rows rows) of every failed
// row in the `pad[0]` word of the tile's first row, so that kStoreFailed CTAs
// of tiles without a failed row read one word and exit.
__global__ void __launch_bounds__(256) select_scan_kernel(SelectRowStats* __restrict__ stats,
                                                         int64_t rows, int Tq, int Tkv,
                                                         int q_pos0, int k_sel, int tile_rows) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const int r = static_cast<int>(row % Tq);
  const int n = min(q_pos0 + r + 1, Tkv);
  if (select_row_failed(stats[row], n, k_sel)) atomicOr(&stats[row - r % tile_rows].pad[0], 1);
}

// Shared memory of the fix-up (rows that did not fail).
constexpr int kFixLists = kSelMaxKeys / 256;  // lists of the longest row
constexpr int kFixBins = 512;                 // 9-bit digits of the candidate keys
constexpr int kFixDigit = 9;
constexpr int kFixLevels = 4;                 // 4 x 9 bits cover a 32-bit key
struct alignas(16) FixupShared {
  uint2 cand[kFixCap + kFixLists];  // the row's lists, each padded to an even length
  int hist[kFixBins];               // histogram of a digit of the candidate keys
  int last[kFixCap];                // columns of the last bin's members (one key value)
  uint32_t bits[kMaxWords];
  int warp_a[kTopkWarps];
  uint64_t bar;                     // completion of the lists' bulk copies
  int abort;
  int neq;
  int sh_digit, sh_above, sh_bin;
};
constexpr uint32_t kNoKey = 0xFFFFFFFFu;  // column of a padding slot

// Rows that did not fail (and rows with n <= k): the k best keys are the sure
// bits plus the need = k - sure best candidates by (score desc, key asc).
// Failed rows are left to select_fallback_kernel.
__global__ void __launch_bounds__(kTopkThreads, 6) select_fixup_kernel(
    const uint32_t* __restrict__ ws, int64_t ws_stride, int64_t sel_words, int64_t cand_off,
    int cand_per_list, int keys_per_chunk, const SelectRowStats* __restrict__ stats, int Tq,
    int Tkv, int q_pos0, int k_sel, int32_t* __restrict__ indices, uint8_t* __restrict__ mask,
    uint32_t* __restrict__ bitmask, int64_t bm_words, int* err) {
  __shared__ FixupShared sh;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t row = blockIdx.x;
  const int n = min(q_pos0 + static_cast<int>(row % Tq) + 1, Tkv);
  const uint32_t* wrow = ws + row * ws_stride;
  int32_t* irow = indices ? indices + row * k_sel : nullptr;
  uint8_t* mrow = mask ? mask + row * k_sel : nullptr;
  uint32_t* brow = bitmask ? bitmask + row * bm_words : nullptr;
  const int nwords = (n + 31) / 32;
  if (n <= k_sel) {  // every key of the row (no score is read)
    const int full = n >> 5, rem_bits = n & 31;
    if (brow)
      for (int64_t w = tid; w < bm_words; w += kTopkThreads)
        brow[w] = w < full ? 0xFFFFFFFFu : (w == full && rem_bits ? (1u << rem_bits) - 1u : 0u);
    for (int s = tid; s < k_sel; s += kTopkThreads) {
      if (irow) irow[s] = min(s, Tkv - 1);  // s itself below n; filler above
      if (mrow) mrow[s] = s < n ? 1 : 0;
    }
    return;
  }
  // the row's counters, sure bits and list counts are read together (one round
  // trip): candidates of every list holding a key of the row, two lists per key
  // chunk (the two interleaved halves), each count <= cand_per_list
  const int nlists = 2 * ((n + keys_per_chunk - 1) / keys_per_chunk);
  const uint2* lists = reinterpret_cast<const uint2*>(wrow + cand_off);
  int c0 = 0, c1 = 0;  // counts of lists 2*tid and 2*tid+1
  if (2 * tid < nlists) c0 = static_cast<int>(wrow[sel_words + 2 * tid]);
  if (2 * tid + 1 < nlists) c1 = static_cast<int>(wrow[sel_words + 2 * tid + 1]);
  for (int w = tid; w < nwords; w += kTopkThreads) sh.bits[w] = wrow[w];
  const SelectRowStats st = stats[row];
  if (select_row_failed(st, n, k_sel)) return;  // select_fallback_kernel's row
  const int need = k_sel - st.sure;  // 0 <= need <= ncand
  if (need <= 0) c0 = c1 = 0;
  const int p0 = (c0 + 1) & ~1, p1 = (c1 + 1) & ~1;  // padded: 16-byte copies
  if (tid == 0) {
    sh.neq = 0;
    sh.abort = 0;
    mbar_init(&sh.bar, 1);
    fence_mbar_init();
  }
  // exclusive scan of the padded counts (nlists <= 2 * kTopkThreads)
  static_assert(kFixLists <= 2 * kTopkThreads, "two lists per thread");
  int incl = p0 + p1;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) sh.warp_a[warp] = incl;
  __syncthreads();
  int before = incl - p0 - p1, total = 0;
#pragma unroll
  for (int w = 0; w < kTopkWarps; ++w) {
    if (w < warp) before += sh.warp_a[w];
    total += sh.warp_a[w];
  }
  if (need > 0) {
    // one bulk copy per non-empty list, all in flight together
    if (p0) bulk_load(&sh.cand[before], lists + static_cast<int64_t>(2 * tid) * cand_per_list,
                      8u * p0, &sh.bar);
    if (p1)
      bulk_load(&sh.cand[before + p0], lists + static_cast<int64_t>(2 * tid + 1) * cand_per_list,
                8u * p1, &sh.bar);
    if (tid == 0) mbar_arrive_expect_tx(&sh.bar, 8u * total);
    if (!mbar_wait(&sh.bar, 0, err, &sh.abort)) {
      mbar_wait_drain(&sh.bar, 0, 200000000LL);  // copies in flight land before the CTA exits
      return;
    }
    // a list of odd length was copied with the slot after its last entry
    if (p0 != c0) sh.cand[before + c0].y = kNoKey;
    if (p1 != c1) sh.cand[before + p0 + c1].y = kNoKey;
  }
  __syncthreads();
  auto set_bit = [&](int j) { atomicOr(&sh.bits[j >> 5], 1u << (j & 31)); };
  if (need > 0 && need >= st.ncand) {
    for (int e = tid; e < total; e += kTopkThreads)
      if (sh.cand[e].y != kNoKey) set_bit(static_cast<int>(sh.cand[e].y));
  } else if (need > 0) {
    // MSB-first radix select of the need-th largest key among the candidates,
    // 9-bit digits of (key - ord_key(lo)) (all candidates lie in [lo, hi]):
    // each level narrows to one digit value, until that bin is taken whole or
    // holds a single key value (4 levels cover 32 bits); higher bins are
    // taken, and the members of a single-value bin tie: the lowest columns win
    uint32_t kmin = ord_key(st.lo), kmax = ord_key(st.hi);
    if (kmin == kNegInfKey) kmin = 0u;          // an open bracket: the whole key range
    if (kmax == 0xFF800000u) kmax = 0xFFFFFFFFu;
    uint32_t lbase[kFixLevels];
    int lsft[kFixLevels], lbin[kFixLevels], nlev = 0, rem = need;
    lbase[0] = kmin;
    lsft[0] = max(0, 32 - __clz(max(kmax - kmin, 1u)) - kFixDigit);
    while (true) {
      for (int bn = tid; bn < kFixBins; bn += kTopkThreads) sh.hist[bn] = 0;
      __syncthreads();
      const int lv = nlev;
      for (int e = tid; e < total; e += kTopkThreads) {
        if (sh.cand[e].y == kNoKey) continue;
        const uint32_t u = ord_key(__uint_as_float(sh.cand[e].x));
        bool in = true;  // in the chosen bin of every level below lv
#pragma unroll
        for (int i = 0; i < kFixLevels; ++i)
          if (i < lv) in = in && static_cast<int>((u - lbase[i]) >> lsft[i]) == lbin[i];
        if (in) atomicAdd(&sh.hist[(u - lbase[lv]) >> lsft[lv]], 1);
      }
      __syncthreads();
      find_threshold_bin<kFixBins>(sh, rem);
      lbin[lv] = sh.sh_digit;
      rem -= sh.sh_above;
      const int cnt = sh.sh_bin;
      nlev = lv + 1;
      if (cnt == rem || lsft[lv] == 0) break;  // the bin is the last
      static_assert(kFixLevels * kFixDigit >= 32, "the last level's digit ends at bit 0");
      lbase[nlev] = lbase[lv] + (static_cast<uint32_t>(lbin[lv]) << lsft[lv]);
      lsft[nlev] = max(0, lsft[lv] - kFixDigit);
    }
    __syncthreads();  // every thread has read the last bin
    const bool whole = sh.sh_bin == rem;  // the last bin is taken whole
    for (int e = tid; e < total; e += kTopkThreads) {
      const uint2 v = sh.cand[e];
      if (v.y == kNoKey) continue;
      const uint32_t u = ord_key(__uint_as_float(v.x));
      int verdict = 0;  // 1 taken, -1 not, 0 member of the last bin
#pragma unroll
      for (int i = 0; i < kFixLevels; ++i) {
        if (i < nlev && verdict == 0) {
          const int bn = static_cast<int>((u - lbase[i]) >> lsft[i]);
          verdict = bn > lbin[i] ? 1 : (bn < lbin[i] ? -1 : 0);
        }
      }
      if (verdict > 0 || (verdict == 0 && whole)) {
        set_bit(static_cast<int>(v.y));
      } else if (verdict == 0) {
        sh.last[atomicAdd(&sh.neq, 1)] = static_cast<int>(v.y);  // <= ncand <= kFixCap
      }
    }
    __syncthreads();
    const int ne = whole ? 0 : sh.neq;
    for (int e = tid; e < ne; e += kTopkThreads) {
      const int j = sh.last[e];
      int rank = 0;  // members with a lower column
      for (int o = 0; o < ne; ++o) rank += sh.last[o] < j ? 1 : 0;
      if (rank < rem) set_bit(j);
    }
  }
  __syncthreads();
  if (brow)
    for (int64_t w = tid; w < bm_words; w += kTopkThreads) brow[w] = w < nwords ? sh.bits[w] : 0u;
  if (irow || mrow) bits_to_lists(sh, nwords, irow, mrow);
}

// Rows whose bracket missed: the plain top-k of their full score rows (written
// into the workspace by the indexer's kStoreFailed pass).  A fixed grid walks
// the rows; CTAs skip rows that did not fail after reading their counters.
template <int kGroups>
__global__ void __launch_bounds__(kTopkThreads) select_fallback_kernel(
    const float* __restrict__ ws, int64_t ws_stride, const SelectRowStats* __restrict__ stats,
    int64_t rows, int Tq, int Tkv, int q_pos0, int k_sel, int32_t* __restrict__ indices,
    uint8_t* __restrict__ mask, uint32_t* __restrict__ bitmask, int64_t bm_words) {
  __shared__ TopkShared<topk_words<kGroups>(), topk_cand_cap<kGroups>()> sh;
  __shared__ int64_t failed[kTopkThreads];
  __shared__ int nfailed;
  // the CTA's rows, kTopkThreads at a time: each thread checks one, the failed
  // ones are listed, then selected one after another by the whole CTA
  for (int64_t r0 = static_cast<int64_t>(blockIdx.x) * kTopkThreads; r0 < rows;
       r0 += static_cast<int64_t>(gridDim.x) * kTopkThreads) {
    if (threadIdx.x == 0) nfailed = 0;
    __syncthreads();
    const int64_t row = r0 + threadIdx.x;
    if (row < rows) {
      const int n = min(q_pos0 + static_cast<int>(row % Tq) + 1, Tkv);
      if (select_row_failed(stats[row], n, k_sel)) failed[atomicAdd(&nfailed, 1)] = row;
    }
    __syncthreads();
    const int nf = nfailed;
    for (int f = 0; f < nf; ++f) {
      const int64_t fr = failed[f];
      const int n = min(q_pos0 + static_cast<int>(fr % Tq) + 1, Tkv);
      topk_row<true, kGroups>(sh, ws + fr * ws_stride, n, Tkv, k_sel, k_sel,
                              indices ? indices + fr * k_sel : nullptr,
                              mask ? mask + fr * k_sel : nullptr,
                              bitmask ? bitmask + fr * bm_words : nullptr, bm_words);
      __syncthreads();  // the next row reuses the shared memory
    }
  }
}

}  // namespace

cudaError_t launch_topk(const float* scores, int64_t score_stride, int B, int Tq, int Tkv,
                        int q_pos0, int k_sel, int k_width, const AdaptiveK& ad,
                        int32_t* indices, uint8_t* mask, uint32_t* bitmask,
                        int64_t bitmask_words, bool finite_rows, cudaStream_t stream) {
  const int64_t rows = static_cast<int64_t>(B) * Tq;
  if (rows == 0) return cudaSuccess;
  auto kernel = finite_rows ? (Tkv >= kLongKeyRange ? topk_kernel<true, kEmitLong>
                                                    : topk_kernel<true, kEmitShort>)
                            : (Tkv >= kLongKeyRange ? topk_kernel<false, kEmitLong>
                                                    : topk_kernel<false, kEmitShort>);
  kernel<<<static_cast<unsigned>(rows), kTopkThreads, 0, stream>>>(
      scores, score_stride, Tq, Tkv, q_pos0, k_sel, k_width, ad, indices, mask, bitmask,
      bitmask_words);
  return cudaGetLastError();
}

cudaError_t launch_row_variance(const float* scores, int64_t score_stride, int B, int Tq, int Tkv,
                                int q_pos0, float* row_var, double* var_sum, cudaStream_t stream) {
  const int64_t rows = static_cast<int64_t>(B) * Tq;
  if (rows == 0) return cudaSuccess;
  row_variance_kernel<<<static_cast<unsigned>(rows), kVarThreads, 0, stream>>>(
      scores, score_stride, Tq, Tkv, q_pos0, row_var);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  var_sum_kernel<<<1, kSumThreads, 0, stream>>>(row_var, rows, var_sum);
  return cudaGetLastError();
}

cudaError_t launch_select_threshold(const float* samples, int64_t stride, int B, int Tq, int Tkv,
                                    int q_pos0, int key_step, int key_off, int k_sel, float z,
                                    SelectRowStats* stats, cudaStream_t stream) {
  const int64_t rows = static_cast<int64_t>(B) * Tq;
  if (rows == 0) return cudaSuccess;
  select_threshold_kernel<<<static_cast<unsigned>((rows + kThrRows - 1) / kThrRows), kTopkThreads,
                            0, stream>>>(samples, stride, rows, Tq, Tkv, q_pos0, key_step, key_off,
                                         k_sel, z, stats);
  return cudaGetLastError();
}

cudaError_t launch_select_scan(SelectRowStats* stats, int B, int Tq, int Tkv, int q_pos0,
                               int k_sel, int tile_rows, cudaStream_t stream) {
  const int64_t rows = static_cast<int64_t>(B) * Tq;
  if (rows == 0) return cudaSuccess;
  select_scan_kernel<<<static_cast<unsigned>((rows + 255) / 256), 256, 0, stream>>>(
      stats, rows, Tq, Tkv, q_pos0, k_sel, tile_rows);
  return cudaGetLastError();
}

cudaError_t launch_select_fixup(const uint32_t* ws, int64_t ws_stride, int64_t sel_words,
                                int64_t cand_off, int cand_per_list, int keys_per_chunk,
                                const SelectRowStats* stats, int B, int Tq, int Tkv, int q_pos0,
                                int k_sel, int32_t* indices, uint8_t* mask, uint32_t* bitmask,
                                int64_t bitmask_words, int* err, cudaStream_t stream) {
  const int64_t rows = static_cast<int64_t>(B) * Tq;
  if (rows == 0) return cudaSuccess;
  select_fixup_kernel<<<static_cast<unsigned>(rows), kTopkThreads, 0, stream>>>(
      ws, ws_stride, sel_words, cand_off, cand_per_list, keys_per_chunk, stats, Tq, Tkv, q_pos0,
      k_sel, indices, mask, bitmask, bitmask_words, err);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  // failed rows: a grid of a few CTAs per SM walks all rows
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const unsigned grid = static_cast<unsigned>(
      std::min<int64_t>((rows + kTopkThreads - 1) / kTopkThreads, 4LL * sms));
  auto fb = Tkv >= kLongKeyRange ? select_fallback_kernel<kEmitLong>
                                 : select_fallback_kernel<kEmitShort>;
  fb<<<grid, kTopkThreads, 0, stream>>>(reinterpret_cast<const float*>(ws), ws_stride, stats,
                                        rows, Tq, Tkv, q_pos0, k_sel, indices, mask, bitmask,
                                        bitmask_words);
  return cudaGetLastError();
}

}  // namespace gsa
