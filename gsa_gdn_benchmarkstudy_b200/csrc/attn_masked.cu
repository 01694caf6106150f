// attn_masked.cu — sparse attention over a per-row selection bitmask on
// tcgen05 tensor cores, with the output gate fused into the epilogue.
//
// Reference: sparse_attention_ref (gsa_ref.py:202-238) gathers, for every
// query row, the k selected key/value rows and runs a masked softmax over
// them; OutputGate (gsa_ref.py:177-180) then multiplies by sigmoid(og).
// Selected keys are distinct (torch.topk returns distinct positions), so
//   softmax over {j selected} (q.k_j * scale)  ==  softmax over all causal j
//   with the logits of unselected keys set to -inf,
// and the product P.V over the full causal key range with P = 0 at
// unselected keys is the same sum.  This kernel therefore streams 128x128
// key tiles of the causal range through the tensor cores (gather-free; the
// selection enters only as 16 bytes of bitmask per row per tile), instead
// of gathering 2*k*H*d bytes per query row as the reference does.
//
// CTA = (batch b, head h, 128-query tile), 12 warps in three warpgroups:
//   warps 0-7  softmax + epilogue.  Warp w serves query rows 32(w%4)..+31
//              (TMEM lane quarter w%4) over the key tiles of parity w/4:
//              even tiles go to warps 0-3, odd tiles to warps 4-7, so each SM
//              sub-partition runs two softmax warps on different tiles with no
//              per-tile synchronisation between them.  Each parity keeps its own
//              running max m, row sum l and TMEM accumulator O_par; the two are
//              merged once in the epilogue.  These warps raise their register
//              budget to kSoftmaxRegs (setmaxnreg) so a whole 128-key row of S
//              stays in registers.
//   warp 8     TMA producer for Q and the K ring (2 stages)
//   warp 9     TMEM owner; one thread issues the QK^T tcgen05.mma
//   warp 10    TMA producer for the V ring (2 stages), so K loads never queue
//              behind V loads
//   warp 11    one thread issues the P.V tcgen05.mma
// Per key tile j (parity par = j % 2):
//   softmax:  load the row of S_j from TMEM into registers and release the S
//             buffer at once (the MMA warp then computes S_{j+2} into it while
//             this tile's exponentials run).  Unselected keys are set to -inf,
//             the tile max t of the selected keys is taken, and the running
//             max is raised lazily: m moves to max(m, t) only when that exceeds
//             m by more than 8/c (c = scale*log2 e), so p = 2^(s*c - m*c) <= 2^8;
//             when it moves, l and this warp's rows of O_par are scaled by
//             2^((m_old - m_new)*c).  P (bf16) goes to shared buffer par in the
//             128B-swizzled K-major layout the MMA reads, once P.V of tile j-2
//             (same buffer, same O_par) has finished.
//   MMA:      S_{j+2} = Q.K_{j+2}^T as soon as S_j is released (warp 9), and
//             O_par += P_j.V_j once P_j is in shared memory (warp 11).
// Epilogue: M = max(m_even, m_odd), O = O_even*2^((m_even-M)c) + O_odd*2^((m_odd-M)c)
//   (likewise l), o = O / l rounded to bf16; optional gate bf16(o * bf16(sigmoid(og))).
//
// TMEM: S0 [0,128), S1 [128,256), O_even [256,384), O_odd [384,512) fp32 columns.
// Shared memory: Q 32 KB, K 2x32 KB, V 2x32 KB, P 2x32 KB + control (one CTA per SM).
#include "kernels.h"

namespace gsa {
namespace {

constexpr int kAtBM = 128;
constexpr int kAtBN = 128;
constexpr int kAtD = 128;
constexpr int kAtTileBytes = kAtBM * kAtD * 2;  // 32 KB: two 128x64 swizzled boxes
constexpr int kAtBoxBytes = kAtTileBytes / 2;   // 16 KB
constexpr int kAtThreads = 384;
constexpr int kAtTmemCols = 512;
constexpr int kAtPairGroup = 4;  // (batch, head) pairs scheduled together, heavy tiles first
constexpr float kRescaleLog2 = 8.0f;            // p may reach 2^8 before m is raised
constexpr long long kDrainCycles = 200000000LL; // ~0.1 s: in-flight copies/MMAs after an abort
// Register split (setmaxnreg): the launch gives 384 threads x 168 registers;
// the control warpgroup drops to kCtrlRegs and the two softmax warpgroups take
// the rest: 128*56 + 256*224 == 384*168.
constexpr int kLaunchRegs = 168;
constexpr int kCtrlRegs = 56;
constexpr int kSoftmaxRegs = 224;
static_assert(128 * kCtrlRegs + 256 * kSoftmaxRegs <= kAtThreads * kLaunchRegs,
              "register split exceeds the launch allocation");

struct AtSmem {
  uint64_t q_full;
  uint64_t k_full[2], v_full[2];
  uint64_t s_full[2];   // S_j computed (also: K stage free)
  uint64_t s_empty[2];  // S_j loaded into registers by the 4 softmax warps
  uint64_t p_full[2];   // P_j written by the 4 softmax warps
  uint64_t p_empty[2];  // P_j.V_j finished (also: V stage and P buffer free)
  uint64_t o_full;
  uint64_t drain[2];    // [issuer] MMAs in flight when the CTA gives up
  uint32_t tmem_base;
  int abort;
  float xm[2][kAtBM];  // [parity][row] running max, for the epilogue merge
  float xl[2][kAtBM];  // [parity][row] row sum
};
// The dynamic shared memory base is 1024-byte aligned (checked at run time),
// so the swizzled tiles need no alignment slack: 7 tiles + the control block.
constexpr int kAtSmemBytes = 7 * kAtTileBytes + ((sizeof(AtSmem) + 15) / 16) * 16;
static_assert(kAtSmemBytes <= 232448, "exceeds 227 KB of shared memory per CTA");

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

template <uint32_t N>
__device__ __forceinline__ void reg_alloc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void reg_dealloc() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

__global__ void __launch_bounds__(kAtThreads, 1)
    masked_attn_kernel(const __grid_constant__ CUtensorMap qmap,
                       const __grid_constant__ CUtensorMap kmap,
                       const __grid_constant__ CUtensorMap vmap, MaskedAttnArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if ((smem_u32(smem_raw) & 1023u) != 0) {  // swizzled TMA/MMA tiles need 1024 B alignment
    if (threadIdx.x == 0) atomicExch(a.err, GSA_ERR_ALIGNMENT);
    return;
  }
  uint8_t* smem = smem_raw;
  uint8_t* q_s = smem;
  uint8_t* k_s = smem + kAtTileBytes;      // 2 stages
  uint8_t* v_s = smem + 3 * kAtTileBytes;  // 2 stages
  uint8_t* p_s = smem + 5 * kAtTileBytes;  // 2 buffers
  AtSmem* sh = reinterpret_cast<AtSmem*>(smem + 7 * kAtTileBytes);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int n_qt = (a.Tq + kAtBM - 1) / kAtBM;
  // Grid (pairs per group, query tiles, groups): the blocks of a group of
  // kAtPairGroup (batch, head) pairs are dispatched heavy tiles first across
  // the whole group, so the last wave holds light tiles, while only the
  // group's K/V (a few MB per pair) is live in L2 at a time.
  const int qt = n_qt - 1 - static_cast<int>(blockIdx.y);
  const int pair = static_cast<int>(blockIdx.z * gridDim.x + blockIdx.x);
  const int h = pair % a.H;
  const int b = pair / a.H;
  const int row0 = qt * kAtBM;
  const int maxpos = a.q_pos0 + min(row0 + kAtBM - 1, a.Tq - 1);
  const int nt = min((a.Tkv + kAtBN - 1) / kAtBN, maxpos / kAtBN + 1);

  if (tid == 0) {
    mbar_init(&sh->q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sh->k_full[s], 1);
      mbar_init(&sh->v_full[s], 1);
      mbar_init(&sh->s_full[s], 1);
      mbar_init(&sh->s_empty[s], 4);
      mbar_init(&sh->p_full[s], 4);
      mbar_init(&sh->p_empty[s], 1);
    }
    mbar_init(&sh->o_full, 1);
    mbar_init(&sh->drain[0], 1);
    mbar_init(&sh->drain[1], 1);
    sh->abort = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(&sh->tmem_base, kAtTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;
  volatile int* abort = &sh->abort;

  if (warp >= 8) {
    reg_dealloc<kCtrlRegs>();
    const int x0 = h * kAtD;
    if (warp == 8 && lane == 0) {
      // ------------------------------------------------ TMA: Q once, K ring
      prefetch_tmap(&qmap);
      prefetch_tmap(&kmap);
      mbar_arrive_expect_tx(&sh->q_full, kAtTileBytes);
      tma_load_3d(q_s, &qmap, x0, row0, b, &sh->q_full);
      tma_load_3d(q_s + kAtBoxBytes, &qmap, x0 + 64, row0, b, &sh->q_full);
      int j = 0;
      for (; j < nt; ++j) {
        const int st = j & 1;
        // stage st is free once S_{j-2} has been computed
        if (!mbar_wait(&sh->s_full[st], ((j >> 1) & 1) ^ 1, a.err, abort)) break;
        uint8_t* kd = k_s + st * kAtTileBytes;
        mbar_arrive_expect_tx(&sh->k_full[st], kAtTileBytes);
        tma_load_3d(kd, &kmap, x0, j * kAtBN, b, &sh->k_full[st]);
        tma_load_3d(kd + kAtBoxBytes, &kmap, x0 + 64, j * kAtBN, b, &sh->k_full[st]);
      }
      if (*abort) {  // let the copies this thread issued land before the CTA exits
        mbar_wait_drain(&sh->q_full, 0, kDrainCycles);
        for (int jj = max(0, j - 2); jj < j; ++jj)
          mbar_wait_drain(&sh->k_full[jj & 1], (jj >> 1) & 1, kDrainCycles);
      }
    } else if (warp == 10 && lane == 0) {
      // ------------------------------------------------ TMA: V ring
      prefetch_tmap(&vmap);
      int j = 0;
      for (; j < nt; ++j) {
        const int st = j & 1;
        // stage st is free once P_{j-2}.V_{j-2} has finished
        if (!mbar_wait(&sh->p_empty[st], ((j >> 1) & 1) ^ 1, a.err, abort)) break;
        uint8_t* vd = v_s + st * kAtTileBytes;
        mbar_arrive_expect_tx(&sh->v_full[st], kAtTileBytes);
        tma_load_3d(vd, &vmap, x0, j * kAtBN, b, &sh->v_full[st]);
        tma_load_3d(vd + kAtBoxBytes, &vmap, x0 + 64, j * kAtBN, b, &sh->v_full[st]);
      }
      if (*abort) {
        for (int jj = max(0, j - 2); jj < j; ++jj)
          mbar_wait_drain(&sh->v_full[jj & 1], (jj >> 1) & 1, kDrainCycles);
      }
    } else if ((warp == 9 || warp == 11) && lane == 0) {
      // ------------------------------------------------ MMA issuers
      // Two threads issue: warp 9 the QK^T MMAs, warp 11 the P.V MMAs.  An
      // issuing thread is held while its MMAs execute, so with one issuer every
      // barrier wait between two batches left the tensor pipe idle.  The two
      // streams touch disjoint TMEM (S buffers / O accumulators), and each
      // thread's tcgen05.commit tracks only its own MMAs.
      constexpr uint32_t idesc_s = idesc_bf16_f32(kAtBM, kAtBN, 0, 0);  // Q, K both K-major
      constexpr uint32_t idesc_o = idesc_bf16_f32(kAtBM, kAtD, 0, 1);   // P K-major, V MN-major
      bool ok = true;
      if (warp == 9) {
        const uint32_t q_base = smem_u32(q_s);
        const uint32_t k_base = smem_u32(k_s);
        ok = mbar_wait(&sh->q_full, 0, a.err, abort);
        // S_j = Q.K_j^T into S buffer j%2, once the softmax has loaded S_{j-2}
        for (int j = 0; ok && j < nt; ++j) {
          const int st = j & 1;
          if (j >= 2 && !(ok = mbar_wait(&sh->s_empty[st], ((j - 2) >> 1) & 1, a.err, abort)))
            break;
          if (!(ok = mbar_wait(&sh->k_full[st], (j >> 1) & 1, a.err, abort))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kAtD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * kAtBoxBytes + (kk & 3) * 32;
            const uint64_t ad = sdesc_sw128(q_base + off, 16, 1024);
            const uint64_t bd = sdesc_sw128(k_base + st * kAtTileBytes + off, 16, 1024);
            tc_mma_ss(tmem + st * kAtBN, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
          }
          tc_commit(&sh->s_full[st]);
        }
      } else {
        const uint32_t v_base = smem_u32(v_s);
        const uint32_t p_base = smem_u32(p_s);
        // O_par += P_j.V_j once the softmax has written P_j
        for (int j = 0; ok && j < nt; ++j) {
          const int st = j & 1;
          const uint32_t ph = (j >> 1) & 1;
          if (!(ok = mbar_wait(&sh->p_full[st], ph, a.err, abort))) break;
          if (!(ok = mbar_wait(&sh->v_full[st], ph, a.err, abort))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kAtBN / 16; ++kk) {
            const uint64_t ad = sdesc_sw128(
                p_base + st * kAtTileBytes + (kk >> 2) * kAtBoxBytes + (kk & 3) * 32, 16, 1024);
            const uint64_t bd =
                sdesc_sw128(v_base + st * kAtTileBytes + kk * 16 * 128, kAtBoxBytes, 1024);
            tc_mma_ss(tmem + (2 + st) * kAtBN, ad, bd, idesc_o, (j > 1 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&sh->p_empty[st]);
        }
        if (ok) tc_commit(&sh->o_full);
      }
      if (!ok) {  // let the MMAs this thread issued finish before TMEM is freed
        uint64_t* d = &sh->drain[warp == 9 ? 0 : 1];
        tc_commit(d);
        mbar_wait_drain(d, 0, kDrainCycles);
      }
    }
  } else {
    reg_alloc<kSoftmaxRegs>();
    // ---------------------------------------------------------- softmax warps
    const int quarter = warp & 3;
    const int par = warp >> 2;           // key-tile parity served by this warp
    const int i = quarter * 32 + lane;   // query row in the tile == TMEM lane
    const int r = row0 + i;
    const bool row_ok = r < a.Tq;
    const int64_t grow = static_cast<int64_t>(b) * a.Tq + r;
    const uint4* bm = reinterpret_cast<const uint4*>(a.bitmask + grow * a.bitmask_words);
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_taddr = tmem + lane_base + par * kAtBN;
    const uint32_t o_taddr = tmem + lane_base + (2 + par) * kAtBN;
    const float c = a.scale * 1.4426950408889634f;
    const uint64_t c2 = f2_pack(c, c);
    const uint32_t pb = smem_u32(p_s) + par * kAtTileBytes;
    bool ok = true;
    float m = -INFINITY;   // running max of this parity (raw dot-product units)
    float l = 0.f;         // row sum of this parity, relative to m
    uint4 bits_next = (row_ok && par < nt) ? bm[par] : make_uint4(0, 0, 0, 0);

    for (int j = par; ok && j < nt; j += 2) {
      const uint32_t ph = (j >> 1) & 1;
      const uint4 bits = bits_next;
      if (row_ok && j + 2 < nt) bits_next = bm[j + 2];
      const uint32_t wb[4] = {bits.x, bits.y, bits.z, bits.w};
      if (!(ok = mbar_wait_warp(&sh->s_full[par], ph, a.err, abort))) break;
      tc_fence_after();
      uint32_t sv[4][32];
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) tmem_ld32(s_taddr + cc * 32, sv[cc]);
      tc_wait_ld();
      // S_j is in registers: hand the buffer back for S_{j+2}
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->s_empty[par]);

      // unselected keys -> -inf; tile max of the selected ones
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float s0 = ((wb[cc] >> e) & 1u) ? __uint_as_float(sv[cc][e]) : -INFINITY;
          const float s1 = ((wb[cc] >> (e + 1)) & 1u) ? __uint_as_float(sv[cc][e + 1]) : -INFINITY;
          sv[cc][e] = __float_as_uint(s0);
          sv[cc][e + 1] = __float_as_uint(s1);
          mx[(e >> 1) & 3] = max3f(mx[(e >> 1) & 3], s0, s1);
        }
      }
      const float tmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      // lazy running max: move only when the tile max exceeds m by more than 8/c
      const float m_old = m;
      const bool raise = tmax > m_old && (m_old == -INFINITY || (tmax - m_old) * c > kRescaleLog2);
      float alpha = 1.f;
      if (raise) {
        alpha = (m_old == -INFINITY) ? 0.f : fast_ex2((m_old - tmax) * c);
        m = tmax;
      }
      const float mc = (m == -INFINITY) ? 0.f : m * c;
      const uint64_t nmc2 = f2_pack(-mc, -mc);

      // p = 2^(s*c - m*c) (0 at unselected keys), row sum, bf16 pack
      uint64_t l2a = 0, l2b = 0;
      uint32_t packed[4][16];
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const uint64_t x2 = f2_fma(
              f2_pack(__uint_as_float(sv[cc][e]), __uint_as_float(sv[cc][e + 1])), c2, nmc2);
          const float p0 = fast_ex2(f2_lo(x2));
          const float p1 = fast_ex2(f2_hi(x2));
          if (e & 2) l2b = f2_add(l2b, f2_pack(p0, p1));
          else l2a = f2_add(l2a, f2_pack(p0, p1));
          packed[cc][e >> 1] = pack_bf16x2(p0, p1);
        }
      }
      const uint64_t l2 = f2_add(l2a, l2b);

      // P buffer par is free (and O_par stable) once P.V of tile j-2 finished
      if (!(ok = mbar_wait_warp(&sh->p_empty[par], ph ^ 1, a.err, abort))) break;
      tc_fence_after();
      // O rows of earlier tiles of this parity follow a raised max (rare)
      if (j >= 2 && __any_sync(0xFFFFFFFFu, raise && m_old != -INFINITY)) {
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
          uint32_t ov[32];
          tmem_ld32(o_taddr + cc * 32, ov);
          tc_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
          tmem_st32(o_taddr + cc * 32, ov);
        }
        tc_wait_st();
      }
      l = l * alpha + (f2_lo(l2) + f2_hi(l2));
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        // keys 32cc..32cc+31 -> box cc/2, 16-byte chunks 4*(cc%2) .. +3 of row i
        const uint32_t box = pb + (cc >> 1) * kAtBoxBytes;
#pragma unroll
        for (int qd = 0; qd < 4; ++qd)
          st_shared_v4(box + sw128_offset(i, (cc & 1) * 4 + qd), packed[cc][4 * qd],
                       packed[cc][4 * qd + 1], packed[cc][4 * qd + 2], packed[cc][4 * qd + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->p_full[par]);  // P_j ready
    }

    // epilogue: merge the two parities, O / l (+ output gate), bf16 store of
    // this warp's 64 output channels (par * 64 ..).  The gates bf16(sigmoid(og))
    // are loaded and computed first, so that their latency overlaps the merge
    // and the wait for the last P.V.
    const uint32_t col0 = par * 64;
    const __nv_bfloat16* grow_p =
        (a.og && row_ok)
            ? static_cast<const __nv_bfloat16*>(a.og) + grow * a.og_stride + h * kAtD + col0
            : nullptr;
    uint32_t gates[32];  // bf16x2: channels (2e, 2e+1)
    if (grow_p) {
      uint4 graw[8];
#pragma unroll
      for (int qd = 0; qd < 8; ++qd) graw[qd] = reinterpret_cast<const uint4*>(grow_p)[qd];
#pragma unroll
      for (int qd = 0; qd < 8; ++qd) {
        const __nv_bfloat16* ge = reinterpret_cast<const __nv_bfloat16*>(&graw[qd]);
#pragma unroll
        for (int e = 0; e < 8; e += 2)
          gates[qd * 4 + (e >> 1)] = pack_bf16x2(sigmoid_ref(__bfloat162float(ge[e])),
                                                 sigmoid_ref(__bfloat162float(ge[e + 1])));
      }
    }
    sh->xm[par][i] = m;
    sh->xl[par][i] = l;
    asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
    const float m_e = sh->xm[0][i], m_o = sh->xm[1][i];
    const float mm = fmaxf(m_e, m_o);
    const float a_e = m_e == -INFINITY ? 0.f : fast_ex2((m_e - mm) * c);
    const float a_o = m_o == -INFINITY ? 0.f : fast_ex2((m_o - mm) * c);
    const float lsum = sh->xl[0][i] * a_e + sh->xl[1][i] * a_o;
    const bool odd_written = nt > 1;  // O_odd is only written when tile 1 exists
    ok = ok && mbar_wait_warp(&sh->o_full, 0, a.err, abort);
    if (ok) {
      tc_fence_after();
      const float inv_l = lsum > 0.f ? 1.0f / lsum : 0.f;
      __nv_bfloat16* orow =
          static_cast<__nv_bfloat16*>(a.out) + grow * a.out_stride + h * kAtD + col0;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        uint32_t oe[32], oo[32];
        tmem_ld32(tmem + lane_base + 2 * kAtBN + col0 + cc * 32, oe);
        if (odd_written) tmem_ld32(tmem + lane_base + 3 * kAtBN + col0 + cc * 32, oo);
        tc_wait_ld();
        if (!row_ok) continue;
#pragma unroll
        for (int e = 0; e < 32; ++e) {  // merged, normalised output (in place)
          float acc = __uint_as_float(oe[e]) * a_e;
          if (odd_written) acc = fmaf(__uint_as_float(oo[e]), a_o, acc);
          oe[e] = __float_as_uint(acc * inv_l);
        }
        const uint32_t* ov = oe;
        uint32_t packed[16];
        if (grow_p) {
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const uint32_t g = gates[cc * 16 + (e >> 1)];
            const float o0 = bf16_round(__uint_as_float(ov[e]));
            const float o1 = bf16_round(__uint_as_float(ov[e + 1]));
            const float g0 = __uint_as_float(g << 16);
            const float g1 = __uint_as_float(g & 0xFFFF0000u);
            packed[e >> 1] = pack_bf16x2(o0 * g0, o1 * g1);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; e += 2)
            packed[e >> 1] = pack_bf16x2(__uint_as_float(ov[e]), __uint_as_float(ov[e + 1]));
        }
        uint4* dst = reinterpret_cast<uint4*>(orow + cc * 32);
#pragma unroll
        for (int qd = 0; qd < 4; ++qd)
          dst[qd] = make_uint4(packed[4 * qd], packed[4 * qd + 1], packed[4 * qd + 2],
                               packed[4 * qd + 3]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, kAtTmemCols);
  }
}

}  // namespace

int masked_attention_regs(int* expected) {
  *expected = kLaunchRegs;
  static std::atomic<int> regs{0};
  int r = regs.load(std::memory_order_acquire);
  if (r == 0) {
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, masked_attn_kernel) != cudaSuccess) return -1;
    r = fa.numRegs;
    regs.store(r, std::memory_order_release);
  }
  return r;
}

cudaError_t launch_masked_attention(const CUtensorMap& qmap, const CUtensorMap& kmap,
                                    const CUtensorMap& vmap, const MaskedAttnArgs& a,
                                    cudaStream_t stream) {
  if (a.B == 0 || a.Tq == 0 || a.Tkv == 0) return cudaSuccess;
  // the setmaxnreg split is valid only for the register count it was written for
  int expected = 0;
  if (masked_attention_regs(&expected) != expected) return cudaErrorNotSupported;
  // once per device; two threads racing here both set the same attribute
  static std::atomic<bool> attr_set[kMaxDevices];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < kMaxDevices && !attr_set[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(masked_attn_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kAtSmemBytes);
    if (e != cudaSuccess) return e;
    attr_set[dev].store(true, std::memory_order_release);
  }
  const int n_qt = (a.Tq + kAtBM - 1) / kAtBM;
  const int pairs = a.B * a.H;
  const int group = pairs % kAtPairGroup == 0 ? kAtPairGroup : (pairs % 2 == 0 ? 2 : 1);
  if (n_qt > 65535 || pairs / group > 65535) return cudaErrorInvalidConfiguration;
  dim3 grid(group, n_qt, pairs / group);
  masked_attn_kernel<<<grid, kAtThreads, kAtSmemBytes, stream>>>(qmap, kmap, vmap, a);
  return cudaGetLastError();
}

}  // namespace gsa
