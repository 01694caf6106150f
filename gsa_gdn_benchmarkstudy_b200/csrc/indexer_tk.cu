// indexer_tk.cu — gated lightning indexer on tcgen05 with keys as the MMA's M
// dimension, and the selection of the fused indexer + top-k in its epilogue.
//
//   score[b,r,j] = sum_h sigmoid(w[b,r,h]) * sigmoid(scale * q[b,r,h,:].k[b,j,:] + bias[h])
//   for j <= q_pos0 + r (causal), -inf above the diagonal.
//
// Reference: GatedLightningIndexer.forward, gsa_ref.py:97-126 (and the Triton
// _fused_gated_indexer_kernel, gsa_opt.py:48-140).  The epilogue evaluates
// sigmoid(z) = 1/2 + tanh(z/2)/2: with hw_h = sigmoid(w_h)/2,
//   score = sum_h hw_h + sum_h hw_h * tanh(dot_h * scale/2 + bias_h/2),
// two scores per f32x2 FMA and one MUFU tanh.approx per score and head.
//
// Layout.  One CTA owns 64 query rows and a chunk of up to 512 keys.  The MMA
// is D[key, (head, row)] = K[key, :] . Q[(head, row), :]: M = 128 keys (TMEM
// lanes), N = 4 heads x 64 rows = 256 columns, K = 64 in four k-steps.  Q
// (4 x [64 rows x 64] bf16, 32 KB) is loaded once by TMA with 128-byte swizzle,
// 128-key tiles of k_I (16 KB) stream through a 4-stage TMA ring, and one
// thread issues four M128 N256 K16 MMAs per tile into one of two 256-column
// TMEM buffers (512 columns: one CTA per SM).  Sixteen epilogue warps: warp w
// reads TMEM lane quarter w%4 (32 consecutive keys, lane = key) and the
// columns of rows [16*(w/4), +16) of every head, so one warp holds 32
// consecutive keys of 16 rows: stores of a row are 128-byte coalesced, and a
// ballot over the warp is one 32-key word of the row's selection bitmask.
//
// Modes (one kernel instance each):
//   kStore       scores of every causal (row, key) pair, -inf above the diagonal
//                inside the chunks it visits (the gsa_indexer_scores path);
//   kSample      scores against a strided subset of the keys (launch key i is
//                sequence key i*key_step + key_off), for the threshold estimate;
//   kSelect      no scores stored: per row, keys scoring above the row's `hi`
//                threshold become bitmask bits, keys in [lo, hi] become
//                candidates (score, key) appended to the row's list, and the
//                number of keys above `hi` is counted;
//   kStoreFailed kStore restricted to rows whose selection failed (their
//                thresholds missed the k-th score or a list overflowed); CTAs
//                without such a row exit at once.
#include "kernels.h"

namespace gsa {
namespace {

constexpr int kTkRows = 64;                  // query rows per CTA
constexpr int kTkKeys = 128;                 // keys per MMA tile (M, TMEM lanes)
constexpr int kTkChunk = 512;                // keys per CTA
constexpr int kTkStages = 4;                 // k_I ring depth
constexpr int kTkHeads = 4;
constexpr int kTkD = 64;
constexpr int kTkN = kTkHeads * kTkRows;     // 256 MMA columns
constexpr int kTkQBytes = kTkN * kTkD * 2;   // 32 KB
constexpr int kTkQBoxBytes = kTkRows * kTkD * 2;  // 8 KB per head
constexpr int kTkKBytes = kTkKeys * kTkD * 2;     // 16 KB per stage
constexpr int kTkTmemCols = 2 * kTkN;        // two accumulator buffers
constexpr int kTkEpiWarps = 16;
constexpr int kTkEpiThreads = 32 * kTkEpiWarps;
constexpr int kTkTmaWarp = kTkEpiWarps;      // warp 16
constexpr int kTkMmaWarp = kTkEpiWarps + 1;  // warp 17: MMA issuer, TMEM owner
constexpr int kTkThreads = 32 * (kTkEpiWarps + 2);
constexpr int kTkWords = kTkChunk / 32;      // bitmask words of a row inside one chunk
constexpr int kTkCandCap = 128;              // candidates of one row staged per CTA
constexpr long long kTkDrainCycles = 200000000LL;
static_assert(kTkRows / 16 * 4 == kTkEpiWarps, "16 rows per epilogue warp, 4 lane quarters");

struct TkCtl {
  uint64_t q_full;
  uint64_t k_full[kTkStages];
  uint64_t k_empty[kTkStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  // per-row parameters, packed so that rows (2p, 2p+1) form one f32x2 operand
  float hw[kTkHeads][kTkRows];  // sigmoid(w)/2
  float hsum[kTkRows];          // sum over heads of hw
  float hi[kTkRows];            // kSelect thresholds
  float lo[kTkRows];
  int pos[kTkRows];             // sequence position of the row, -1 beyond Tq
  int skip[kTkRows];            // kStoreFailed: 1 = the row's scores are not stored
};

struct TkSel {
  uint32_t bits[kTkRows][kTkWords];
  uint2 cand[kTkRows][kTkCandCap];
  int cand_cnt[kTkRows];
  int sure[4][kTkRows];         // per lane quarter: no two warps add to one counter
};

constexpr int align_up(int x, int a) { return (x + a - 1) / a * a; }
constexpr int kTkCtlBytes = align_up(static_cast<int>(sizeof(TkCtl)), 128);
template <int kMode>
constexpr int tk_smem_bytes() {
  return 1024 + kTkQBytes + kTkStages * kTkKBytes + kTkCtlBytes +
         (kMode == kIdxSelect ? align_up(static_cast<int>(sizeof(TkSel)), 128) : 0);
}
static_assert(tk_smem_bytes<kIdxSelect>() <= 227 * 1024, "shared memory budget");

__device__ __forceinline__ void epi_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(kTkEpiThreads) : "memory");
}

template <int kMode>
__global__ void __launch_bounds__(kTkThreads, 1)
    indexer_tk_kernel(const __grid_constant__ CUtensorMap qmap,
                      const __grid_constant__ CUtensorMap kmap, IndexerTkArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* q_s = smem;
  uint8_t* k_s = smem + kTkQBytes;
  TkCtl* sh = reinterpret_cast<TkCtl*>(k_s + kTkStages * kTkKBytes);
  TkSel* sel = reinterpret_cast<TkSel*>(reinterpret_cast<uint8_t*>(sh) + kTkCtlBytes);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int n_rb = (a.Tq + kTkRows - 1) / kTkRows;
  const int rb = n_rb - 1 - static_cast<int>(blockIdx.y);  // heavy row blocks first
  const int kc = blockIdx.x;
  const int b = blockIdx.z;
  const int row0 = rb * kTkRows;
  const int maxpos = a.q_pos0 + min(row0 + kTkRows - 1, a.Tq - 1);
  // launch keys i with position i*key_step + key_off <= maxpos
  const int key_end = maxpos < a.key_off ? 0 : min((maxpos - a.key_off) / a.key_step + 1, a.nkeys);
  const int key0 = kc * kTkChunk;
  if (key0 >= key_end) return;  // chunk entirely above the diagonal
  const int ntiles = (min(kTkChunk, key_end - key0) + kTkKeys - 1) / kTkKeys;
  const int64_t row_base = static_cast<int64_t>(b) * a.Tq + row0;  // global row of r = 0

  if constexpr (kMode == kIdxStoreFailed) {
    bool failed = false;
    if (tid < kTkRows && row0 + tid < a.Tq) {
      const int n = min(a.q_pos0 + row0 + tid + 1, a.Tkv);
      failed = select_row_failed(a.stats[row_base + tid], n, a.k_sel);
    }
    if (!__syncthreads_or(failed)) return;
  }

  // ---- per-row parameters and (kSelect) staging areas
  if (tid < kTkRows) {
    const int r = tid;
    const bool ok = row0 + r < a.Tq;
    float hs = 0.f;
#pragma unroll
    for (int h = 0; h < kTkHeads; ++h) {
      float wv = 0.f;
      if (ok)
        wv = __bfloat162float(static_cast<const __nv_bfloat16*>(a.w)[(row_base + r) * a.w_stride + h]);
      const float hw = 0.5f * sigmoid_ref(wv);
      sh->hw[h][r] = hw;
      hs += hw;
    }
    sh->hsum[r] = hs;
    sh->pos[r] = ok ? a.q_pos0 + row0 + r : -1;
    if constexpr (kMode == kIdxSelect) {
      sh->hi[r] = ok ? a.stats[row_base + r].hi : 0.f;
      sh->lo[r] = ok ? a.stats[row_base + r].lo : 0.f;
    }
    if constexpr (kMode == kIdxStoreFailed) {
      sh->skip[r] = 1;
      if (ok) {
        const int n = min(a.q_pos0 + row0 + r + 1, a.Tkv);
        sh->skip[r] = select_row_failed(a.stats[row_base + r], n, a.k_sel) ? 0 : 1;
      }
    }
  }
  if constexpr (kMode == kIdxSelect) {
    uint32_t* z = &sel->bits[0][0];
    for (int i = tid; i < kTkRows * kTkWords; i += kTkThreads) z[i] = 0u;
    for (int i = tid; i < kTkRows; i += kTkThreads) sel->cand_cnt[i] = 0;
    for (int i = tid; i < 4 * kTkRows; i += kTkThreads) (&sel->sure[0][0])[i] = 0;
  }
  if (tid == 0) {
    mbar_init(&sh->q_full, 1);
    for (int s = 0; s < kTkStages; ++s) {
      mbar_init(&sh->k_full[s], 1);
      mbar_init(&sh->k_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sh->acc_full[s], 1);
      mbar_init(&sh->acc_empty[s], kTkEpiWarps);
    }
    mbar_init(&sh->drain, 1);
    sh->abort = 0;
    fence_mbar_init();
  }
  if (warp == kTkMmaWarp) {
    tmem_alloc(&sh->tmem_base, kTkTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;
  volatile int* abort = &sh->abort;

  if (warp == kTkTmaWarp) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&qmap);
      prefetch_tmap(&kmap);
      mbar_arrive_expect_tx(&sh->q_full, kTkQBytes);
      for (int h = 0; h < kTkHeads; ++h)
        tma_load_3d(q_s + h * kTkQBoxBytes, &qmap, h * kTkD, row0, b, &sh->q_full);
      int s = 0;
      for (; s < ntiles; ++s) {
        const int st = s % kTkStages;
        if (!mbar_wait(&sh->k_empty[st], ((s / kTkStages) & 1) ^ 1, a.err, abort)) break;
        mbar_arrive_expect_tx(&sh->k_full[st], kTkKBytes);
        tma_load_3d(k_s + st * kTkKBytes, &kmap, 0, key0 + s * kTkKeys, b, &sh->k_full[st]);
      }
      if (*abort) {  // let the copies this thread issued land before the CTA exits
        mbar_wait_drain(&sh->q_full, 0, kTkDrainCycles);
        for (int ss = max(0, s - kTkStages); ss < s; ++ss)
          mbar_wait_drain(&sh->k_full[ss % kTkStages], (ss / kTkStages) & 1, kTkDrainCycles);
      }
    }
  } else if (warp == kTkMmaWarp) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kTkKeys, kTkN, 0, 0);
      const uint32_t q_base = smem_u32(q_s);
      const uint32_t k_base = smem_u32(k_s);
      bool ok = mbar_wait(&sh->q_full, 0, a.err, abort);
      for (int s = 0; ok && s < ntiles; ++s) {
        const int st = s % kTkStages;
        const int buf = s & 1;
        if (!(ok = mbar_wait(&sh->k_full[st], (s / kTkStages) & 1, a.err, abort))) break;
        if (!(ok = mbar_wait(&sh->acc_empty[buf], ((s >> 1) & 1) ^ 1, a.err, abort))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kTkD / 16; ++kk) {
          const uint64_t ad = sdesc_sw128(k_base + st * kTkKBytes + kk * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(q_base + kk * 32, 16, 1024);
          tc_mma_ss(tmem + buf * kTkN, ad, bd, idesc, kk > 0 ? 1u : 0u);
        }
        tc_commit(&sh->k_empty[st]);
        tc_commit(&sh->acc_full[buf]);
      }
      if (!ok) {  // let the MMAs this thread issued finish before TMEM is freed
        tc_commit(&sh->drain);
        mbar_wait_drain(&sh->drain, 0, kTkDrainCycles);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------ epilogue (warps 0-15)
    const int qd = warp & 3;   // TMEM lane quarter: keys [32*qd, +32) of a tile
    const int rg = warp >> 2;  // rows [16*rg, +16)
    const uint32_t lane_base = static_cast<uint32_t>(qd * 32) << 16;
    const uint32_t lt_mask = (1u << lane) - 1u;
    const uint64_t hs2 = f2_pack(0.5f * a.scale, 0.5f * a.scale);
    uint64_t hb2[kTkHeads];
#pragma unroll
    for (int h = 0; h < kTkHeads; ++h) hb2[h] = f2_pack(0.5f * a.bias[h], 0.5f * a.bias[h]);
    const float kNegInf = -__int_as_float(0x7F800000);

    for (int s = 0; s < ntiles; ++s) {
      const int buf = s & 1;
      if (!mbar_wait_warp(&sh->acc_full[buf], (s >> 1) & 1, a.err, abort)) break;
      tc_fence_after();
      const int i = key0 + s * kTkKeys + qd * 32 + lane;  // launch key of this lane
      const int jpos = i * a.key_step + a.key_off;       // its sequence position
      const bool in_range = i < key_end;
      // two halves of the warp's 16 rows, 8 TMEM columns per head each; the
      // buffer is released once the second half is in registers
#pragma unroll
      for (int half = 0; half < 2; ++half) {
      uint32_t raw[kTkHeads][8];
#pragma unroll
      for (int h = 0; h < kTkHeads; ++h)
        tmem_ld8(tmem + lane_base + buf * kTkN + h * kTkRows + rg * 16 + half * 8, raw[h]);
      tc_wait_ld();
      if (half == 1) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh->acc_empty[buf]);
      }
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const int r = rg * 16 + half * 8 + 2 * p;
        uint64_t acc2 = *reinterpret_cast<const uint64_t*>(&sh->hsum[r]);
#pragma unroll
        for (int h = 0; h < kTkHeads; ++h) {
          const uint64_t z2 = f2_fma(
              f2_pack(__uint_as_float(raw[h][2 * p]), __uint_as_float(raw[h][2 * p + 1])), hs2,
              hb2[h]);
          const uint64_t t2 = f2_pack(fast_tanh(f2_lo(z2)), fast_tanh(f2_hi(z2)));
          acc2 = f2_fma(t2, *reinterpret_cast<const uint64_t*>(&sh->hw[h][r]), acc2);
        }
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int rr = r + e;
          const float sc = e ? f2_hi(acc2) : f2_lo(acc2);
          const int pr = sh->pos[rr];
          if constexpr (kMode == kIdxSelect) {
            const bool valid = in_range && jpos <= pr;
            const float hi = sh->hi[rr], lo = sh->lo[rr];
            const bool gt = valid && !(sc <= hi);  // NaN counts as above, as it ranks first
            const bool ca = valid && !gt && sc >= lo;
            const uint32_t gb = __ballot_sync(0xFFFFFFFFu, gt);
            const uint32_t cb = __ballot_sync(0xFFFFFFFFu, ca);
            if (lane == 0) {
              sel->bits[rr][s * 4 + qd] = gb;
              sel->sure[qd][rr] += __popc(gb);
            }
            if (cb) {
              int base = 0;
              if (lane == 0) base = atomicAdd(&sel->cand_cnt[rr], __popc(cb));
              base = __shfl_sync(0xFFFFFFFFu, base, 0);
              const int c = base + __popc(cb & lt_mask);
              if (ca && c < kTkCandCap)
                sel->cand[rr][c] = make_uint2(__float_as_uint(sc), static_cast<uint32_t>(jpos));
            }
          } else {
            bool store = pr >= 0 && in_range;
            if constexpr (kMode == kIdxStoreFailed) store = store && !sh->skip[rr];
            if constexpr (kMode == kIdxSample) store = store && jpos <= pr;
            if (store)
              a.out[(row_base + rr) * a.out_stride + i] = jpos <= pr ? sc : kNegInf;
          }
        }
      }
      }
    }

    if constexpr (kMode == kIdxSelect) {
      // ---- flush: bitmask words, counts and candidate lists of the 64 rows
      epi_bar();
      if (!*abort) {
        const int wfirst = key0 / 32;
        for (int e = tid; e < kTkRows * kTkWords; e += kTkEpiThreads) {
          const int r = e / kTkWords, w = e % kTkWords;
          if (row0 + r < a.Tq && wfirst + w < a.bitmask_words)
            a.sel_bits[(row_base + r) * a.sel_stride + wfirst + w] = sel->bits[r][w];
        }
        if (tid < kTkRows && row0 + tid < a.Tq) {
          const int total = sel->sure[0][tid] + sel->sure[1][tid] + sel->sure[2][tid] +
                            sel->sure[3][tid];
          if (total) atomicAdd(&a.stats[row_base + tid].sure, total);
        }
        for (int r = warp; r < kTkRows; r += kTkEpiWarps) {
          if (row0 + r >= a.Tq) continue;
          SelectRowStats* st = &a.stats[row_base + r];
          int n = sel->cand_cnt[r];
          if (n > kTkCandCap) {
            if (lane == 0) atomicOr(&st->flags, kSelOverflow);
            continue;
          }
          if (n == 0) continue;
          int base = 0;
          if (lane == 0) base = atomicAdd(&st->ncand, n);
          base = __shfl_sync(0xFFFFFFFFu, base, 0);
          if (base + n > a.cand_cap) {
            if (lane == 0) atomicOr(&st->flags, kSelOverflow);
            continue;
          }
          uint2* dst = reinterpret_cast<uint2*>(a.sel_bits + (row_base + r) * a.sel_stride +
                                                a.bitmask_words) + base;
          for (int c = lane; c < n; c += 32) dst[c] = sel->cand[r][c];
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kTkMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTkTmemCols);
  }
}

template <int kMode>
cudaError_t launch_mode(const CUtensorMap& qmap, const CUtensorMap& kmap, const IndexerTkArgs& a,
                        cudaStream_t stream) {
  // once per device; two threads racing here both set the same attribute
  static std::atomic<bool> attr_set[kMaxDevices];
  int dev = 0;
  cudaGetDevice(&dev);
  constexpr int smem = tk_smem_bytes<kMode>();
  if (dev >= 0 && dev < kMaxDevices && !attr_set[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(indexer_tk_kernel<kMode>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_set[dev].store(true, std::memory_order_release);
  }
  const int n_rb = (a.Tq + kTkRows - 1) / kTkRows;
  const int n_kc = (a.nkeys + kTkChunk - 1) / kTkChunk;
  if (n_rb > 65535 || a.B > 65535) return cudaErrorInvalidConfiguration;
  dim3 grid(n_kc, n_rb, a.B);
  indexer_tk_kernel<kMode><<<grid, kTkThreads, smem, stream>>>(qmap, kmap, a);
  return cudaGetLastError();
}

}  // namespace

int indexer_tk_rows_per_cta() { return kTkRows; }
int indexer_tk_keys_per_tile() { return kTkKeys; }

cudaError_t launch_indexer_tk(int mode, const CUtensorMap& qmap, const CUtensorMap& kmap,
                              const IndexerTkArgs& a, cudaStream_t stream) {
  if (a.B == 0 || a.Tq == 0 || a.nkeys == 0) return cudaSuccess;
  switch (mode) {
    case kIdxStore: return launch_mode<kIdxStore>(qmap, kmap, a, stream);
    case kIdxSample: return launch_mode<kIdxSample>(qmap, kmap, a, stream);
    case kIdxSelect: return launch_mode<kIdxSelect>(qmap, kmap, a, stream);
    case kIdxStoreFailed: return launch_mode<kIdxStoreFailed>(qmap, kmap, a, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace gsa
