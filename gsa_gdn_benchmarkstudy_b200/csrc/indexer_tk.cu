// indexer_tk.cu — the tcgen05 gated lightning indexer, and the selection of
// the fused indexer + top-k in its epilogue.
//
//   score[b,r,j] = sum_h sigmoid(w[b,r,h]) * sigmoid(scale * q[b,r,h,:].k[b,j,:] + bias[h])
//   for j <= q_pos0 + r (causal), -inf above the diagonal.
//
// Reference: GatedLightningIndexer.forward, gsa_ref.py:97-126 (fp32 math on
// bf16-rounded projections; einsum, *scale, +bias, sigmoid, *sigmoid(w), sum
// over heads, masked_fill(-inf)), and the Triton _fused_gated_indexer_kernel
// of gsa_opt.py:48-140.  The epilogue evaluates sigmoid(z) = 1/2 + tanh(z/2)/2:
// with hw_h = sigmoid(w_h)/2,
//   score = sum_h hw_h + sum_h hw_h * tanh(dot_h * scale/2 + bias_h/2),
// two keys per f32x2 FMA and one MUFU tanh.approx per key and head (the
// cheapest logistic on this SM: one MUFU op and two FMAs).  Scores come out
// about 1e-5 (relative) from the reference's separately rounded fp32 ops.
//
// Layout.  One CTA owns 128 query rows and a chunk of up to 512 keys; only
// chunks at or below the diagonal run.  Q (4 heads x [128 x 64] bf16) is loaded
// once by TMA with 128-byte swizzle; 32-key sub-tiles of k_I stream through a
// 4-stage TMA ring.  Per sub-tile one thread issues 4 heads x 4 k-steps of
// tcgen05.mma (M=128 rows, N=32 keys, K=16) into one of two TMEM accumulator
// buffers (4 heads x 32 fp32 columns each; 256 columns per CTA, two CTAs per
// SM).  Eight epilogue warps, two per TMEM lane quarter: thread = query row =
// TMEM lane, each warp of a pair takes 16 of the 32 key columns.  A thread
// therefore holds 16 consecutive scores of its own row, with the row's gate
// weights and thresholds in registers.
//
// Modes (one kernel instance each):
//   kStore       scores of every causal (row, key) pair, -inf above the diagonal
//                inside the chunks it visits (gsa_indexer_scores);
//   kSample      scores against a strided subset of the keys (launch key i is
//                sequence key i*key_step + key_off), for the threshold estimate;
//   kSelect      no scores stored: a key scoring above its row's `hi` threshold
//                becomes a bit of the row's bitmask, a key in [lo, hi] becomes a
//                candidate (score, key) in the row's list of this chunk half;
//                counts of both go to the row's SelectRowStats;
//   kStoreFailed kStore restricted to rows whose selection failed (the bracket
//                missed the k-th score or a list overflowed); CTAs without such
//                a row exit at once.
#include "kernels.h"

namespace gsa {
namespace {

constexpr int kIdxBM = 128;      // query rows per CTA
constexpr int kIdxBN = 32;       // keys per MMA sub-tile
constexpr int kIdxChunk = 512;   // keys per CTA
// kStoreFailed CTAs take 4096 keys each: the launch is mostly CTAs that read
// one flag and exit, and fewer of them cost less
template <int kMode>
constexpr int idx_chunk() { return kMode == kIdxStoreFailed ? 4096 : kIdxChunk; }
constexpr int kIdxStages = 4;    // K ring depth
constexpr int kIdxHeads = 4;
constexpr int kIdxD = 64;
constexpr int kIdxQBytes = kIdxBM * kIdxD * 2;    // 16 KB per head
constexpr int kIdxKBytes = kIdxBN * kIdxD * 2;    // 4 KB per stage
constexpr int kIdxTmemCols = 256;                 // 2 buffers x 4 heads x 32
constexpr int kIdxEpiWarps = 8;                   // two per TMEM lane quarter, 16 columns each
constexpr int kIdxEpiThreads = 32 * kIdxEpiWarps;
constexpr int kIdxTmaWarp = kIdxEpiWarps;         // warp 8: TMA producer
constexpr int kIdxMmaWarp = kIdxEpiWarps + 1;     // warp 9: MMA issuer, TMEM owner
constexpr int kIdxThreads = 32 * (kIdxEpiWarps + 2);
constexpr long long kIdxDrainCycles = 200000000LL;  // ~0.1 s after an abort
constexpr int kIdxWords = kIdxChunk / 32;           // bitmask words of a row in one chunk
constexpr int kIdxBitsPitch = kIdxWords + 1;        // padded: lanes (rows) hit distinct banks

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
constexpr int kIdxCtlBytes = 256;
static_assert(sizeof(IdxSmem) <= kIdxCtlBytes, "control block exceeds its slot");
// kStore / kSample write their scores with TMA: each epilogue warp stages
// its 32 rows x 16 keys of a sub-tile (fp32, 64-byte rows, 64B swizzle) and
// stores the box in one bulk copy, so a row's keys reach L2 as whole
// sectors instead of 16 bytes per row per warp store instruction.
template <int kMode>
constexpr bool idx_tma_store() { return kMode == kIdxStore || kMode == kIdxSample; }
constexpr int kIdxBoxBytes = 32 * 16 * 4;  // one warp's staging box
template <int kMode>
constexpr int idx_staging_bytes() { return idx_tma_store<kMode>() ? kIdxEpiWarps * kIdxBoxBytes : 0; }
template <int kMode>
constexpr int idx_smem_bytes() {
  return 1024 /*align slack*/ + kIdxHeads * kIdxQBytes + kIdxStages * kIdxKBytes +
         idx_staging_bytes<kMode>() + kIdxCtlBytes +
         (kMode == kIdxSelect ? kIdxBM * kIdxBitsPitch * 4 : 0);
}

// Byte offset of 16-byte chunk c (0..3) of row r in a box of 64-byte rows
// with the TMA 64-byte swizzle (chunk index XOR bits 1-2 of the row).
__device__ __forceinline__ uint32_t sw64_offset(uint32_t r, uint32_t c) {
  return r * 64u + ((c ^ ((r >> 1) & 3u)) << 4);
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, int x, int y, int z,
                                             const void* smem_src) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(z), "r"(smem_u32(smem_src))
               : "memory");
}

__device__ __forceinline__ void epi_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(kIdxEpiThreads) : "memory");
}

template <int kMode>
__global__ void __launch_bounds__(kIdxThreads, 2)
    indexer_tk_kernel(const __grid_constant__ CUtensorMap qmap,
                      const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap omap, IndexerTkArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* q_s = smem;                                   // 4 x 16 KB
  uint8_t* k_s = smem + kIdxHeads * kIdxQBytes;          // 4 x 4 KB
  uint8_t* staging = k_s + kIdxStages * kIdxKBytes;       // 1024-byte aligned
  IdxSmem* sh = reinterpret_cast<IdxSmem*>(staging + idx_staging_bytes<kMode>());
  uint32_t* bits_s = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(sh) + kIdxCtlBytes);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int n_qt = (a.Tq + kIdxBM - 1) / kIdxBM;
  const int qt = n_qt - 1 - static_cast<int>(blockIdx.y);  // heavy tiles first
  const int kc = blockIdx.x;
  const int b = blockIdx.z;
  const int row0 = qt * kIdxBM;
  const int maxpos = a.q_pos0 + min(row0 + kIdxBM - 1, a.Tq - 1);
  // launch keys i whose sequence position i*key_step + key_off is <= maxpos
  const int key_end =
      maxpos < a.key_off ? 0 : min((maxpos - a.key_off) / a.key_step + 1, a.nkeys);
  constexpr int kChunk = idx_chunk<kMode>();
  const int key0 = kc * kChunk;
  if (key0 >= key_end) return;  // chunk entirely above the diagonal
  const int nsub = (min(kChunk, key_end - key0) + kIdxBN - 1) / kIdxBN;
  const int64_t row_base = static_cast<int64_t>(b) * a.Tq + row0;  // global row of tile row 0

  if constexpr (kMode == kIdxStoreFailed) {
    if (a.stats[row_base].pad[0] == 0) return;  // no row of this tile failed
  }
  if constexpr (kMode == kIdxSelect) {
    for (int i = tid; i < kIdxBM * kIdxBitsPitch; i += kIdxThreads) bits_s[i] = 0u;
  }

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
    const int64_t grow = row_base + i;
    const int pos = a.q_pos0 + r;
    // keys of the row: launch keys j with j*key_step + key_off <= pos and j < nkeys
    const int jlim = (!row_ok || pos < a.key_off)
                         ? 0
                         : min((pos - a.key_off) / a.key_step + 1, a.nkeys);
    // sigmoid(z) = 1/2 + tanh(z/2)/2, so with hw_h = sigmoid(w_h)/2:
    //   score = sum_h hw_h + sum_h hw_h * tanh(dot_h * scale/2 + bias_h/2)
    float hw[kIdxHeads], hb[kIdxHeads], hsum = 0.f;
#pragma unroll
    for (int h = 0; h < kIdxHeads; ++h) {
      float wv = 0.f;
      if (row_ok)
        wv = __bfloat162float(static_cast<const __nv_bfloat16*>(a.w)[grow * a.w_stride + h]);
      hw[h] = 0.5f * sigmoid_ref(wv);
      hb[h] = 0.5f * a.bias[h];
      hsum += hw[h];
    }
    const float hscale = 0.5f * a.scale;
    bool store_row = row_ok;
    if constexpr (kMode == kIdxStoreFailed)
      store_row = row_ok && select_row_failed(a.stats[grow], min(pos + 1, a.Tkv), a.k_sel);
    float hi = 0.f, lo = 0.f;
    int sure = 0, ncand = 0;
    uint2* slots = nullptr;
    if constexpr (kMode == kIdxSelect) {
      if (row_ok) {
        hi = a.stats[grow].hi;
        lo = a.stats[grow].lo;
      }
      slots = reinterpret_cast<uint2*>(a.sel_bits + grow * a.sel_stride + a.cand_off) +
              static_cast<int64_t>(2 * kc + half) * a.cand_per_list;
    }
    float* orow = a.out + grow * a.out_stride;
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
      const int j0 = key0 + s * kIdxBN + half * kCols;  // launch key of acc[0]
      if constexpr (kMode == kIdxSelect) {
        // keys above hi -> bits; keys in [lo, hi] -> candidates (NaN ranks first: a bit)
        const int nvalid = min(max(jlim - j0, 0), kCols);
        const uint32_t vmask = (1u << nvalid) - 1u;
        uint32_t mg = 0u, ml = 0u;
#pragma unroll
        for (int e = 0; e < kCols; ++e) {
          mg |= static_cast<uint32_t>(!(acc[e] <= hi)) << e;
          ml |= static_cast<uint32_t>(acc[e] >= lo) << e;
        }
        mg &= vmask;
        const uint32_t mc = ml & ~mg & vmask;
        sure += __popc(mg);
        reinterpret_cast<uint16_t*>(bits_s + i * kIdxBitsPitch + s)[half] =
            static_cast<uint16_t>(mg);
        if (mc) {
          if (ncand + __popc(mc) <= a.cand_per_list) {
#pragma unroll
            for (int e = 0; e < kCols; ++e)
              if (mc & (1u << e))
                slots[ncand++] =
                    make_uint2(__float_as_uint(acc[e]), static_cast<uint32_t>(j0 + e));
          } else {
            ncand = a.cand_per_list + 1;  // overflow: the row takes the exact fallback
          }
        }
      } else if constexpr (idx_tma_store<kMode>()) {
        if constexpr (kMode == kIdxStore) {
#pragma unroll
          for (int e = 0; e < kCols; ++e)
            if (j0 + e >= jlim) acc[e] = -INFINITY;
        }
        // this warp's box: rows (its lanes) x keys [j0, j0 + 16); TMA clips
        // rows past Tq and keys past the launch's last key
        uint8_t* box = staging + warp * kIdxBoxBytes;
        if (s > 0 && lane == 0)  // the previous store has read the box
          asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        __syncwarp();
        const uint32_t bx = smem_u32(box);
#pragma unroll
        for (int c = 0; c < 4; ++c)
          asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(bx + sw64_offset(lane, c)),
                       "f"(acc[4 * c]), "f"(acc[4 * c + 1]), "f"(acc[4 * c + 2]),
                       "f"(acc[4 * c + 3])
                       : "memory");
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_3d(&omap, j0, row0 + (warp & 3) * 32, b, box);
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
      } else if (store_row) {
        if constexpr (kMode == kIdxStoreFailed) {
#pragma unroll
          for (int e = 0; e < kCols; ++e)
            if (j0 + e >= jlim) acc[e] = -INFINITY;
        }
        if (j0 + kCols <= a.nkeys) {
          float4* dst = reinterpret_cast<float4*>(orow + j0);
#pragma unroll
          for (int v = 0; v < kCols / 4; ++v)
            dst[v] = make_float4(acc[4 * v], acc[4 * v + 1], acc[4 * v + 2], acc[4 * v + 3]);
        } else {
#pragma unroll
          for (int e = 0; e < kCols; ++e)
            if (j0 + e < a.nkeys) orow[j0 + e] = acc[e];
        }
      }
    }

    if constexpr (idx_tma_store<kMode>()) {
      // the stores of this warp are complete before its shared memory goes
      if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
      __syncwarp();
    }
    if constexpr (kMode == kIdxSelect) {
      // ---- flush: the tile's bitmask words, then each row's counters
      epi_bar();
      if (!*abort) {
        const int wfirst = key0 / 32;
        for (int e = tid; e < kIdxBM * kIdxWords; e += kIdxEpiThreads) {
          const int rr = e / kIdxWords, w = e % kIdxWords;
          if (row0 + rr < a.Tq && wfirst + w < a.bitmask_words)
            a.sel_bits[(row_base + rr) * a.sel_stride + wfirst + w] =
                bits_s[rr * kIdxBitsPitch + w];
        }
        if (row_ok) {
          SelectRowStats* st = &a.stats[grow];
          a.sel_bits[grow * a.sel_stride + a.bitmask_words + 2 * kc + half] =
              static_cast<uint32_t>(ncand);
          if (sure) atomicAdd(&st->sure, sure);
          const int kept = min(ncand, a.cand_per_list);
          if (kept) atomicAdd(&st->ncand, kept);
          if (ncand > a.cand_per_list) atomicOr(&st->flags, kSelOverflow);
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

template <int kMode>
cudaError_t launch_mode(const CUtensorMap& qmap, const CUtensorMap& kmap,
                        const CUtensorMap& omap, const IndexerTkArgs& a,
                        cudaStream_t stream) {
  // once per device; two threads racing here both set the same attribute
  static std::atomic<bool> attr_set[kMaxDevices];
  int dev = 0;
  cudaGetDevice(&dev);
  constexpr int smem = idx_smem_bytes<kMode>();
  if (dev >= 0 && dev < kMaxDevices && !attr_set[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(indexer_tk_kernel<kMode>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_set[dev].store(true, std::memory_order_release);
  }
  const int n_qt = (a.Tq + kIdxBM - 1) / kIdxBM;
  const int n_kc = (a.nkeys + idx_chunk<kMode>() - 1) / idx_chunk<kMode>();
  if (n_qt > 65535 || a.B > 65535) return cudaErrorInvalidConfiguration;
  dim3 grid(n_kc, n_qt, a.B);
  indexer_tk_kernel<kMode><<<grid, kIdxThreads, smem, stream>>>(qmap, kmap, omap, a);
  return cudaGetLastError();
}

}  // namespace

int indexer_tk_rows_per_cta() { return kIdxBM; }
int indexer_tk_keys_per_tile() { return kIdxBN; }
int indexer_tk_keys_per_cta() { return kIdxChunk; }

cudaError_t launch_indexer_tk(int mode, const CUtensorMap& qmap, const CUtensorMap& kmap,
                              const CUtensorMap& omap,
                              const IndexerTkArgs& a, cudaStream_t stream) {
  if (a.B == 0 || a.Tq == 0 || a.nkeys == 0) return cudaSuccess;
  switch (mode) {
    case kIdxStore: return launch_mode<kIdxStore>(qmap, kmap, omap, a, stream);
    case kIdxSample: return launch_mode<kIdxSample>(qmap, kmap, omap, a, stream);
    case kIdxSelect: return launch_mode<kIdxSelect>(qmap, kmap, omap, a, stream);
    case kIdxStoreFailed: return launch_mode<kIdxStoreFailed>(qmap, kmap, omap, a, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace gsa
