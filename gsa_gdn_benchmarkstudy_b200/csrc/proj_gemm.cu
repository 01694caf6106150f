// proj_gemm.cu — the fused projection GEMM with RoPE and the value gate in
// its epilogue (bf16 in, fp32 accumulation in TMEM, bf16 out).
//
// Reference: the mega-GEMM of gsa_opt.py:582-609 (x times the concatenated
// q, k, v, value-gate, output-gate and indexer weights, biases added) and the
// track_B element-wise work that follows it (gsa_opt.py:683-696): the value
// gate v * sigmoid(vg) (ValueGate, gsa_ref.py:163-166) and RoPE on q and k
// (apply_rotary_pos_emb, gsa_ref.py:29-40).  Here those run in the GEMM's
// epilogue, on the accumulator tile while it is still on chip, so neither the
// raw q/k/v/vg columns nor a separate element-wise pass over them touch HBM.
// The output gate's sigmoid stays with the attention epilogue, which consumes
// the og logits (attn_masked.cu).
//
// Packed weight (built by gsa_fused_projection_pack): rows in 256-row column
// tiles, so that every tile's epilogue has what it needs on chip:
//   tiles [0, D/256)            q, two heads per tile      -> RoPE  -> q_out
//   tiles [D/256, D/128)        k, two heads per tile      -> RoPE  -> k_out
//   tiles [D/128, D/128 + D/128) v channels 128i..+127 then vg channels
//                               128i..+127                 -> gate  -> v_out
//   then ceil(R/256) tiles      og | iq | ik | iw | zeros  -> +bias -> rest
// with R = D + H_I*d_I + d_I + H_I the width of the rest columns.
//
// Rounding follows the unfused path (torch addmm, then the element-wise ops in
// the module dtype): every projection is bf16(acc + bias); RoPE is
// bf16(bf16(x1*c1) + bf16(-x2*s1)) and bf16(bf16(x2*c2) + bf16(x1*s2)) with x
// the rounded projection; the gate is bf16(v * bf16(sigmoid(vg))).  Products
// of two bf16 values are exact in fp32.
//
// Kernel: persistent, clusters of two CTAs (one per SM).  A cluster computes
// 256x256 output tiles with tcgen05.mma.cta_group::2 (M=256, N=256, K=16):
// each CTA holds 128 rows of x and 128 of the tile's 256 weight rows in its
// shared memory, and 128 rows x 256 fp32 columns of the accumulator in its
// TMEM.  Per CTA, ten warps:
//   warp 0     TMA producer: a 5-stage ring of (x 128x64, w 128x64) tiles; its
//              copies signal the leader CTA's stage barrier (cta_group::2
//              form, no multicast: every CTA loads only its own halves)
//   warp 1     TMEM owner (512 columns: two 256-column accumulators); in the
//              leader CTA one thread issues the MMAs and commits them to both
//              CTAs' barriers
//   warps 2-9  epilogue: TMEM lane quarter warp%4, one output row per thread,
//              two warps per quarter splitting each tile's columns; results go
//              through 128B-swizzled shared staging boxes (32 rows x 64
//              columns) to TMA stores
// The two accumulators let the epilogue of tile i run while the MMAs of tile
// i+1 proceed.  Every mbarrier wait is bounded; on expiry the kernel records
// GSA_ERR_DEVICE_TIMEOUT and every role stops.
#include "kernels.h"

namespace gsa {
namespace {

#ifndef GSA_PG_STAGES
#define GSA_PG_STAGES 5
#endif
#ifndef GSA_PG_BOXES
#define GSA_PG_BOXES 2
#endif
#ifndef GSA_PG_HINTS
#define GSA_PG_HINTS 1
#endif
constexpr int kPgBM = 128;            // rows per CTA (256 per cluster)
constexpr int kPgBN = 256;            // output columns per tile
constexpr int kPgBK = 64;             // K per stage (128-byte rows)
constexpr int kPgStages = GSA_PG_STAGES;
constexpr int kPgHalfBytes = kPgBM * kPgBK * 2;   // 16 KB: x rows or weight rows of one CTA
constexpr int kPgStageBytes = 2 * kPgHalfBytes;   // 32 KB
constexpr int kPgEpiWarps = 8;                     // two per TMEM lane quarter
constexpr int kPgThreads = 64 + 32 * kPgEpiWarps;  // producer, MMA/TMEM, epilogue
constexpr int kPgBoxBytes = 32 * 128;             // staging box: 32 rows x 64 bf16
constexpr int kPgBoxesPerWarp = GSA_PG_BOXES;     // staging boxes per epilogue warp
static_assert(kPgBoxesPerWarp >= 2 && kPgBoxesPerWarp <= 4, "staging boxes per warp");
constexpr int kPgStagingBytes = kPgEpiWarps * kPgBoxesPerWarp * kPgBoxBytes;
// L2 policy of the loads and stores: the packed weight is read once per
// 256-row block of x and is kept (evict_last); outputs are written once and
// not read back by this kernel (evict_first).
constexpr bool kPgHints = GSA_PG_HINTS != 0;
constexpr long long kPgDrainCycles = 200000000LL;

struct PgSmem {
  uint64_t full[kPgStages];    // [leader] both CTAs' halves of a stage landed
  uint64_t empty[kPgStages];   // stage consumed by the MMAs (committed to both CTAs)
  uint64_t acc_full[2];        // accumulator b complete (committed to both CTAs)
  uint64_t acc_empty[2];       // [leader] both CTAs' epilogues read accumulator b
  uint64_t drain;              // [leader] MMAs in flight when the cluster gives up
  uint32_t tmem_base;
  int abort;
};
constexpr int kPgSmemBytes =
    kPgStages * kPgStageBytes + kPgStagingBytes + ((sizeof(PgSmem) + 127) / 128) * 128;
static_assert(kPgSmemBytes <= 232448, "exceeds 227 KB of shared memory per CTA");

// ------------------------------------------------------------ cluster helpers
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The shared::cluster address of the same object in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(saddr), "r"(rank));
  return d;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 2-D tile load into this CTA's shared memory whose completion is counted on
// `bar_cluster` (the leader CTA's stage barrier).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, int x,
                                                 int y, uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}
// The same with an L2 eviction policy (createpolicy).
__device__ __forceinline__ void tma_load_2d_pair_hint(void* smem_dst, const CUtensorMap* map,
                                                      int x, int y, uint32_t bar_cluster,
                                                      uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int x, int y,
                                             const void* smem_src, uint64_t policy) {
  if (kPgHints)
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint"
        " [%0, {%1, %2}], [%3], %4;" ::"l"(reinterpret_cast<uint64_t>(map)),
        "r"(x), "r"(y), "r"(smem_u32(smem_src)), "l"(policy)
        : "memory");
  else
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y), "r"(smem_u32(smem_src))
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until at most n (0..3) committed store groups still read shared memory.
__device__ __forceinline__ void bulk_wait_read(int n) {
  switch (n) {
    case 0: asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.bulk.wait_group.read 2;" ::: "memory"); break;
    default: asm volatile("cp.async.bulk.wait_group.read 3;" ::: "memory"); break;
  }
}
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// tcgen05, cluster-pair forms.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_mma_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on `bar` (same offset) in both CTAs of the pair when all MMAs
// this thread issued so far have finished.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar) {
  const uint16_t mask = 3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(mask)
      : "memory");
}

__device__ __forceinline__ float bf(float x) { return bf16_round(x); }

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

// 8 bf16 values of a 16-byte global load as floats.
__device__ __forceinline__ void unpack8(const uint4 u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// Per-warp epilogue state: the warp's staging boxes (a ring of
// kPgBoxesPerWarp), its row slab and its TMEM lane quarter.  A box is taken
// with acquire(), filled by the warp and stored with release(), which commits
// one store group; at most two boxes are taken and not yet released.
struct Epi {
  uint8_t* boxes;
  int acq;              // boxes taken so far
  int rel;              // boxes released (store groups committed) so far
  int lane;
  int row0;             // first global row of this warp's 32-row slab
  uint32_t tl;          // TMEM address of this warp's lane quarter, column 0
  uint64_t policy;      // L2 policy of the stores

  // The next box, once the store that last read it has read it: that store
  // is group acq - kPgBoxesPerWarp, so rel - (acq - kPgBoxesPerWarp + 1)
  // later groups may still be pending.
  __device__ __forceinline__ uint8_t* acquire() {
    uint8_t* b = boxes + (acq % kPgBoxesPerWarp) * kPgBoxBytes;
    if (acq >= kPgBoxesPerWarp && lane == 0)
      bulk_wait_read(max(0, rel - (acq - kPgBoxesPerWarp + 1)));
    __syncwarp();
    ++acq;
    return b;
  }
  // Store a filled box at output columns [x0, x0 + 64) of this warp's slab.
  __device__ __forceinline__ void release(const uint8_t* b, const CUtensorMap* map, int x0) {
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(map, x0, row0, b, policy);
      bulk_commit();
    }
    ++rel;
  }
};

// 8 values -> 16-byte chunk `chunk` of this lane's row in a staging box.
__device__ __forceinline__ void put8(const uint8_t* box, int lane, int chunk, const float (&y)[8]) {
  st_shared_v4(smem_u32(box) + sw128_offset(lane, chunk), pack_bf16x2(y[0], y[1]),
               pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]), pack_bf16x2(y[6], y[7]));
}

// The two epilogue warps of a TMEM lane quarter split every tile: `half`
// selects a head of a q/k tile, 64 of the 128 channels of a v/vg tile, or
// two of the four boxes of a rest tile.

// q or k tile, head `half`: x1 = channels 0..63, x2 = 64..127 of the head;
// out1 = x1*c1 - x2*s1, out2 = x2*c2 + x1*s2 (rotate_half).
__device__ __forceinline__ void epi_rope(Epi& e, uint32_t acc, const CUtensorMap* map, int col0,
                                         const __nv_bfloat16* crow, const __nv_bfloat16* srow,
                                         int half) {
  uint8_t* s1b = e.acquire();
  uint8_t* s2b = e.acquire();
  const uint32_t h0 = acc + 128 * half;
#pragma unroll 1
  for (int j0 = 0; j0 < 64; j0 += 32) {
    uint4 cs[4][4];  // cos / sin chunks of this thread's row, loaded before the TMEM wait
#pragma unroll
    for (int blk = 0; blk < 4; ++blk) {
      const int j = j0 + 8 * blk;
      cs[blk][0] = *reinterpret_cast<const uint4*>(crow + j);
      cs[blk][1] = *reinterpret_cast<const uint4*>(crow + 64 + j);
      cs[blk][2] = *reinterpret_cast<const uint4*>(srow + j);
      cs[blk][3] = *reinterpret_cast<const uint4*>(srow + 64 + j);
    }
    uint32_t x1[32], x2[32];
    tmem_ld32(e.tl + h0 + j0, x1);
    tmem_ld32(e.tl + h0 + 64 + j0, x2);
    tc_wait_ld();
#pragma unroll
    for (int blk = 0; blk < 4; ++blk) {
      const int j = j0 + 8 * blk;
      float c1[8], c2[8], s1[8], s2[8];
      unpack8(cs[blk][0], c1);
      unpack8(cs[blk][1], c2);
      unpack8(cs[blk][2], s1);
      unpack8(cs[blk][3], s2);
      float y1[8], y2[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float a = bf(__uint_as_float(x1[8 * blk + i]));
        const float b = bf(__uint_as_float(x2[8 * blk + i]));
        y1[i] = bf(__fadd_rn(bf(__fmul_rn(a, c1[i])), bf(__fmul_rn(-b, s1[i]))));
        y2[i] = bf(__fadd_rn(bf(__fmul_rn(b, c2[i])), bf(__fmul_rn(a, s2[i]))));
      }
      put8(s1b, e.lane, j / 8, y1);
      put8(s2b, e.lane, j / 8, y2);
    }
  }
  e.release(s1b, map, col0 + 128 * half);
  e.release(s2b, map, col0 + 128 * half + 64);
}

// v/vg tile: columns 0..127 are v, 128..255 the matching vg logits (bias
// added): out = v * bf16(sigmoid(vg)), channels 64*half .. +63.
__device__ __forceinline__ void epi_gate(Epi& e, uint32_t acc, const CUtensorMap* map, int col0,
                                         const float* vg_bias, int half) {
  uint8_t* s = e.acquire();
#pragma unroll 1
  for (int c0 = 64 * half; c0 < 64 * half + 64; c0 += 32) {
    uint32_t va[32], ga[32];
    tmem_ld32(e.tl + acc + c0, va);
    tmem_ld32(e.tl + acc + 128 + c0, ga);
    tc_wait_ld();
#pragma unroll
    for (int blk = 0; blk < 4; ++blk) {
      const float4 b0 = *reinterpret_cast<const float4*>(vg_bias + c0 + 8 * blk);
      const float4 b1 = *reinterpret_cast<const float4*>(vg_bias + c0 + 8 * blk + 4);
      const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
      float y[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float v = bf(__uint_as_float(va[8 * blk + i]));
        const float g = bf(__fadd_rn(__uint_as_float(ga[8 * blk + i]), bb[i]));
        y[i] = bf(__fmul_rn(v, bf(sigmoid_ref(g))));
      }
      put8(s, e.lane, (c0 % 64) / 8 + blk, y);
    }
  }
  e.release(s, map, col0 + 64 * half);
}

// Rest tile (og | iq | ik | iw): out = acc + bias, boxes 2*half and
// 2*half + 1; boxes at or past `nbox_valid` (the zero padding) are not stored.
__device__ __forceinline__ void epi_plain(Epi& e, uint32_t acc, const CUtensorMap* map, int col0,
                                          const float* bias, int nbox_valid, int half) {
#pragma unroll 1
  for (int k = 2 * half; k < min(2 * half + 2, nbox_valid); ++k) {
    uint8_t* s = e.acquire();
    const int cb = 64 * k;
#pragma unroll 1
    for (int c = 0; c < 64; c += 32) {
      uint32_t xa[32];
      tmem_ld32(e.tl + acc + cb + c, xa);
      tc_wait_ld();
#pragma unroll
      for (int blk = 0; blk < 4; ++blk) {
        const float4 b0 = *reinterpret_cast<const float4*>(bias + cb + c + 8 * blk);
        const float4 b1 = *reinterpret_cast<const float4*>(bias + cb + c + 8 * blk + 4);
        const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        float y[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = __fadd_rn(__uint_as_float(xa[8 * blk + i]), bb[i]);
        put8(s, e.lane, c / 8 + blk, y);
      }
    }
    e.release(s, map, col0 + cb);
  }
}

__global__ void __launch_bounds__(kPgThreads, 1)
    proj_gemm_kernel(const __grid_constant__ CUtensorMap xmap,
                     const __grid_constant__ CUtensorMap wmap,
                     const __grid_constant__ CUtensorMap qmap,
                     const __grid_constant__ CUtensorMap kmap,
                     const __grid_constant__ CUtensorMap vmap,
                     const __grid_constant__ CUtensorMap rmap, ProjGemmArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  // Every CTA of a cluster takes the same branch here (same shared layout),
  // so a misaligned base ends both before the cluster barrier.
  if ((smem_u32(smem_raw) & 1023u) != 0) {
    if (tid == 0) atomicExch(a.err, GSA_ERR_ALIGNMENT);
    return;
  }
  uint8_t* stages = smem_raw;
  uint8_t* staging = smem_raw + kPgStages * kPgStageBytes;
  PgSmem* sh = reinterpret_cast<PgSmem*>(staging + kPgStagingBytes);

  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int npairs = static_cast<int>(gridDim.x >> 1);
  const int m_tiles = (a.M + 2 * kPgBM - 1) / (2 * kPgBM);
  const int total = m_tiles * a.n_tiles;
  const int nk = a.K / kPgBK;

  if (tid == 0) {
    for (int s = 0; s < kPgStages; ++s) {
      mbar_init(&sh->full[s], 1);
      mbar_init(&sh->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sh->acc_full[b], 1);
      mbar_init(&sh->acc_empty[b], 2 * kPgEpiWarps);
    }
    mbar_init(&sh->drain, 1);
    sh->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(&sh->tmem_base, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // the peer's barriers and TMEM exist before anyone signals them
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;
  volatile int* abort = &sh->abort;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    prefetch_tmap(&xmap);
    prefetch_tmap(&wmap);
    const uint64_t keep_w = kPgHints ? policy_evict_last() : 0;
    int it = 0;
    bool ok = true;
    for (int tile = pair; ok && tile < total; tile += npairs) {
      const int m = tile / a.n_tiles, n = tile % a.n_tiles;
      const int xrow = m * 2 * kPgBM + static_cast<int>(rank) * kPgBM;
      const int wrow = n * kPgBN + static_cast<int>(rank) * kPgBM;
      for (int kb = 0; kb < nk; ++kb, ++it) {
        const int s = it % kPgStages;
        if (!(ok = mbar_wait(&sh->empty[s], ((it / kPgStages) & 1) ^ 1, a.err, abort))) break;
        const uint32_t full_leader = map_to_rank(smem_u32(&sh->full[s]), 0);
        if (leader) mbar_arrive_expect_tx(&sh->full[s], 2 * kPgStageBytes);
        uint8_t* st = stages + s * kPgStageBytes;
        tma_load_2d_pair(st, &xmap, kb * kPgBK, xrow, full_leader);
        if (kPgHints)
          tma_load_2d_pair_hint(st + kPgHalfBytes, &wmap, kb * kPgBK, wrow, full_leader, keep_w);
        else
          tma_load_2d_pair(st + kPgHalfBytes, &wmap, kb * kPgBK, wrow, full_leader);
      }
    }
  } else if (warp == 1 && lane == 0 && leader) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = idesc_bf16_f32(2 * kPgBM, kPgBN, 0, 0);  // both K-major
    int it = 0, lt = 0;
    bool ok = true;
    for (int tile = pair; ok && tile < total; tile += npairs, ++lt) {
      const int b = lt & 1;
      if (!(ok = mbar_wait(&sh->acc_empty[b], ((lt >> 1) & 1) ^ 1, a.err, abort))) break;
      tc_fence_after();
      for (int kb = 0; kb < nk; ++kb, ++it) {
        const int s = it % kPgStages;
        if (!(ok = mbar_wait(&sh->full[s], (it / kPgStages) & 1, a.err, abort))) break;
        tc_fence_after();
        const uint32_t xs = smem_u32(stages + s * kPgStageBytes);
        const uint32_t ws = xs + kPgHalfBytes;
#pragma unroll
        for (int kk = 0; kk < kPgBK / 16; ++kk) {
          const uint64_t ad = sdesc_sw128(xs + kk * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(ws + kk * 32, 16, 1024);
          tc_mma_pair(tmem + b * kPgBN, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
        }
        tc_commit_pair(&sh->empty[s]);
      }
      if (ok) tc_commit_pair(&sh->acc_full[b]);
    }
    if (!ok) {  // let the MMAs issued so far finish before TMEM is freed
      tc_commit_pair(&sh->drain);
      mbar_wait_drain(&sh->drain, 0, kPgDrainCycles);
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;  // warps 2-5 and 6-9 split each tile
    Epi e;
    e.boxes = staging + (warp - 2) * kPgBoxesPerWarp * kPgBoxBytes;
    e.acq = 0;
    e.rel = 0;
    e.lane = lane;
    e.policy = kPgHints ? policy_evict_first() : 0;
    e.tl = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t acc_empty0 = map_to_rank(smem_u32(&sh->acc_empty[0]), 0);
    const uint32_t acc_empty1 = map_to_rank(smem_u32(&sh->acc_empty[1]), 0);
    const int qt = a.q_tiles, vt = a.v_tiles;
    int lt = 0;
    bool ok = true;
    for (int tile = pair; ok && tile < total; tile += npairs, ++lt) {
      const int m = tile / a.n_tiles, n = tile % a.n_tiles;
      const int b = lt & 1;
      if (!(ok = mbar_wait_warp(&sh->acc_full[b], (lt >> 1) & 1, a.err, abort))) break;
      tc_fence_after();
      e.row0 = m * 2 * kPgBM + static_cast<int>(rank) * kPgBM + quarter * 32;
      if (e.row0 < a.M) {
        const uint32_t acc = static_cast<uint32_t>(b * kPgBN);
        if (n < 2 * qt) {
          const int g = min(e.row0 + lane, a.M - 1);
          const int64_t t = a.pos0 + g % a.T;
          epi_rope(e, acc, n < qt ? &qmap : &kmap, (n % qt) * kPgBN, a.cos + t * 128,
                   a.sin + t * 128, half);
        } else if (n < 2 * qt + vt) {
          epi_gate(e, acc, &vmap, (n - 2 * qt) * 128, a.bias + n * kPgBN + 128, half);
        } else {
          const int box0 = (n - 2 * qt - vt) * 4;
          epi_plain(e, acc, &rmap, box0 * 64, a.bias + n * kPgBN, min(4, a.rest_boxes - box0),
                    half);
        }
      }
      // this warp's reads of accumulator b are done
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(b ? acc_empty1 : acc_empty0);
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  __syncthreads();
  if (*abort && tid == 0) {
    // copies this CTA issued may still be landing: give them time (bounded)
    const long long t0 = clock64();
    while (clock64() - t0 < 20000000LL) {
    }
  }
  tc_fence_before();
  cluster_sync_all();  // the leader's MMAs and the peer's arrivals are over
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

}  // namespace

int proj_gemm_max_clusters() {
  static std::atomic<int> cached[kMaxDevices];
  static std::atomic<bool> attr_set[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
  if (!attr_set[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(proj_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kPgSmemBytes) != cudaSuccess ||
        cudaFuncSetAttribute(proj_gemm_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed,
                             0) != cudaSuccess)
      return 0;
    attr_set[dev].store(true, std::memory_order_release);
  }
  int c = cached[dev].load(std::memory_order_acquire);
  if (c > 0) return c;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(sms / 2 * 2));
  cfg.blockDim = dim3(kPgThreads);
  cfg.dynamicSmemBytes = kPgSmemBytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaOccupancyMaxActiveClusters(&c, proj_gemm_kernel, &cfg) != cudaSuccess || c <= 0)
    return 0;
  cached[dev].store(c, std::memory_order_release);
  return c;
}

cudaError_t launch_proj_gemm(const CUtensorMap& xmap, const CUtensorMap& wmap,
                             const CUtensorMap& qmap, const CUtensorMap& kmap,
                             const CUtensorMap& vmap, const CUtensorMap& rmap,
                             const ProjGemmArgs& a, int clusters, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * clusters));
  cfg.blockDim = dim3(kPgThreads);
  cfg.dynamicSmemBytes = kPgSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, proj_gemm_kernel, xmap, wmap, qmap, kmap, vmap, rmap, a);
}

}  // namespace gsa
