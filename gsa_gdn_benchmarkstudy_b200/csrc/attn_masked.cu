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
// CTA = (batch b, head h, 128-query tile).  Warp roles:
//   warps 0-7  softmax + epilogue.  Warp w serves query rows 32(w%4)..+31
//              (TMEM lane quarter w%4) over the key tiles of parity w/4:
//              even tiles go to warps 0-3, odd tiles to warps 4-7, so each SM
//              sub-partition runs two softmax warps on different tiles with no
//              per-tile synchronisation between them.  Each parity keeps its own
//              running max m, row sum l and TMEM accumulator O_par; the two are
//              merged once in the epilogue.
//   warp 8     TMA producer (Q once; K and V 128x128 tiles, 2-stage rings)
//   warp 9     TMEM owner + single-thread tcgen05.mma issuer
// Per key tile j (parity par = j % 2):
//   MMA:      S_j = Q.K_j^T into TMEM S buffer par (issued one tile ahead);
//             O_par += P_j.V_j once P_j is in shared memory.
//   softmax:  p = 2^(s*c - m*c), c = scale*log2(e), for selected keys, using the
//             running max m of this parity without waiting for the tile max.
//             m is raised only when some selected s*c - m*c exceeds 8 (p > 256):
//             then the warp recomputes the tile's p from S with the new m and
//             scales l and its rows of O_par by 2^((m_old - m_new)*c); the P.V of
//             the previous tile of the same parity has finished by then.  A
//             row's first selected keys set m from an exact tile max.
//             P (bf16) goes to shared buffer par in the 128B-swizzled K-major
//             layout the MMA reads.
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
constexpr int kAtThreads = 320;
constexpr int kAtTmemCols = 512;
constexpr float kRescaleP = 256.0f;             // p may reach 2^8 before m is raised

struct AtSmem {
  uint64_t q_full;
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2], s_empty[2];
  uint64_t p_full[2], p_empty[2];
  uint64_t o_full;
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

// Masked max of this thread's row of one S tile (raw dot-product units).
__device__ __forceinline__ float row_tile_max(uint32_t s_taddr, const uint32_t (&wb)[4]) {
  float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll 1
  for (int cc = 0; cc < 4; ++cc) {
    uint32_t sv[32];
    tmem_ld32(s_taddr + cc * 32, sv);
    tc_wait_ld();
#pragma unroll
    for (int e = 0; e < 32; ++e)
      if ((wb[cc] >> e) & 1u) mx[e & 3] = fmaxf(mx[e & 3], __uint_as_float(sv[e]));
  }
  return fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
}

// One pass over this thread's row of an S tile: p = 2^(s*c - m*c) for the
// selected keys (0 elsewhere) goes, as bf16, into row i of the swizzled P
// tile at pb.  Returns the row sum of p; `over` is set when some p exceeds
// kRescaleP (the running max m must then be raised).
__device__ __forceinline__ float row_exp_pass(uint32_t s_taddr, const uint32_t (&wb)[4], float c,
                                              float m, uint32_t pb, int i, bool& over) {
  const float mc = (m == -INFINITY) ? 0.f : m * c;
  const uint64_t c2 = f2_pack(c, c), nmc2 = f2_pack(-mc, -mc);
  uint64_t l2a = 0, l2b = 0;  // packed partial row sums
  uint32_t pmax = 0;          // packed bf16 max of p (p >= 0)
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    uint32_t sv[32];
    tmem_ld32(s_taddr + cc * 32, sv);
    tc_wait_ld();
    uint32_t packed[16];
#pragma unroll
    for (int e = 0; e < 32; e += 2) {
      const uint64_t x2 =
          f2_fma(f2_pack(__uint_as_float(sv[e]), __uint_as_float(sv[e + 1])), c2, nmc2);
      const float p0 = ((wb[cc] >> e) & 1u) ? fast_ex2(f2_lo(x2)) : 0.f;
      const float p1 = ((wb[cc] >> (e + 1)) & 1u) ? fast_ex2(f2_hi(x2)) : 0.f;
      if (e & 2) l2b = f2_add(l2b, f2_pack(p0, p1));
      else l2a = f2_add(l2a, f2_pack(p0, p1));
      packed[e >> 1] = pack_bf16x2(p0, p1);
      pmax = bf2_max(pmax, packed[e >> 1]);
    }
    // keys 32cc..32cc+31 -> box cc/2, 16-byte chunks 4*(cc%2) .. +3 of row i
    const uint32_t box = pb + (cc >> 1) * kAtBoxBytes;
#pragma unroll
    for (int qd = 0; qd < 4; ++qd)
      st_shared_v4(box + sw128_offset(i, (cc & 1) * 4 + qd), packed[4 * qd], packed[4 * qd + 1],
                   packed[4 * qd + 2], packed[4 * qd + 3]);
  }
  const float pm = fmaxf(__uint_as_float(pmax << 16), __uint_as_float(pmax & 0xFFFF0000u));
  over = pm > kRescaleP;
  const uint64_t l2 = f2_add(l2a, l2b);
  return f2_lo(l2) + f2_hi(l2);
}

struct RowState {
  float m, l, lt;
};

// Rare path, kept out of line so the hot loop is not duplicated: rows whose p
// overshot raise m to the exact tile max; l and this warp's O rows (earlier
// tiles of the same parity) are scaled by 2^((m_old - m_new) c); then the
// tile's p are recomputed.  All lanes of the warp call it together.
__device__ __noinline__ RowState row_rescale_redo(uint32_t s_taddr, uint32_t o_taddr, uint32_t w0,
                                                  uint32_t w1, uint32_t w2, uint32_t w3, float c,
                                                  float m, float l, bool over, int j,
                                                  uint32_t pb, int i) {
  const uint32_t wb[4] = {w0, w1, w2, w3};
  const float tm = row_tile_max(s_taddr, wb);
  float alpha = 1.f;
  if (over) {
    alpha = fast_ex2((m - tm) * c);
    m = tm;
  }
  l *= alpha;
  if (j >= 2) {  // O of this parity holds P.V of earlier tiles
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
  bool over2;
  const float lt = row_exp_pass(s_taddr, wb, c, m, pb, i, over2);
  return RowState{m, l, lt};
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
  const int qt = n_qt - 1 - static_cast<int>(blockIdx.x);  // heavy tiles first
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int row0 = qt * kAtBM;
  const int maxpos = a.q_pos0 + min(row0 + kAtBM - 1, a.Tq - 1);
  const int nt = min((a.Tkv + kAtBN - 1) / kAtBN, maxpos / kAtBN + 1);

  if (tid == 0) {
    mbar_init(&sh->q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sh->k_full[s], 1);
      mbar_init(&sh->k_empty[s], 1);
      mbar_init(&sh->v_full[s], 1);
      mbar_init(&sh->v_empty[s], 1);
      mbar_init(&sh->s_full[s], 1);
      mbar_init(&sh->s_empty[s], 4);
      mbar_init(&sh->p_full[s], 4);
      mbar_init(&sh->p_empty[s], 1);
    }
    mbar_init(&sh->o_full, 1);
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

  if (warp == 8) {
    // ---------------------------------------------------------- TMA producer
    if (lane == 0) {
      prefetch_tmap(&qmap);
      prefetch_tmap(&kmap);
      prefetch_tmap(&vmap);
      const int x0 = h * kAtD;
      mbar_arrive_expect_tx(&sh->q_full, kAtTileBytes);
      tma_load_3d(q_s, &qmap, x0, row0, b, &sh->q_full);
      tma_load_3d(q_s + kAtBoxBytes, &qmap, x0 + 64, row0, b, &sh->q_full);
      for (int j = 0; j < nt; ++j) {
        const int st = j & 1;
        const uint32_t ph = ((j >> 1) & 1) ^ 1;
        if (!mbar_wait(&sh->k_empty[st], ph, a.err, abort)) break;
        uint8_t* kd = k_s + st * kAtTileBytes;
        mbar_arrive_expect_tx(&sh->k_full[st], kAtTileBytes);
        tma_load_3d(kd, &kmap, x0, j * kAtBN, b, &sh->k_full[st]);
        tma_load_3d(kd + kAtBoxBytes, &kmap, x0 + 64, j * kAtBN, b, &sh->k_full[st]);
        if (!mbar_wait(&sh->v_empty[st], ph, a.err, abort)) break;
        uint8_t* vd = v_s + st * kAtTileBytes;
        mbar_arrive_expect_tx(&sh->v_full[st], kAtTileBytes);
        tma_load_3d(vd, &vmap, x0, j * kAtBN, b, &sh->v_full[st]);
        tma_load_3d(vd + kAtBoxBytes, &vmap, x0 + 64, j * kAtBN, b, &sh->v_full[st]);
      }
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(kAtBM, kAtBN, 0, 0);  // Q, K both K-major
      constexpr uint32_t idesc_o = idesc_bf16_f32(kAtBM, kAtD, 0, 1);   // P K-major, V MN-major
      const uint32_t q_base = smem_u32(q_s);
      const uint32_t k_base = smem_u32(k_s);
      const uint32_t v_base = smem_u32(v_s);
      const uint32_t p_base = smem_u32(p_s);
      bool ok = mbar_wait(&sh->q_full, 0, a.err, abort);

      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&sh->k_full[st], ph, a.err, abort)) return false;
        if (!mbar_wait(&sh->s_empty[st], ph ^ 1, a.err, abort)) return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kAtD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kAtBoxBytes + (kk & 3) * 32;
          const uint64_t ad = sdesc_sw128(q_base + off, 16, 1024);
          const uint64_t bd = sdesc_sw128(k_base + st * kAtTileBytes + off, 16, 1024);
          tc_mma_ss(tmem + st * kAtBN, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
        tc_commit(&sh->s_full[st]);
        tc_commit(&sh->k_empty[st]);
        return true;
      };

      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < nt; ++j) {
        if (j + 1 < nt && !(ok = issue_s(j + 1))) break;
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&sh->v_full[st], ph, a.err, abort)) { ok = false; break; }
        if (!mbar_wait(&sh->p_full[st], ph, a.err, abort)) { ok = false; break; }
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
        tc_commit(&sh->v_empty[st]);
      }
      if (ok) tc_commit(&sh->o_full);
    }
    __syncwarp();
  } else {
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
      // a row's first selected keys: start m from the exact tile max
      if (__any_sync(0xFFFFFFFFu, row_ok && m == -INFINITY)) {
        const float tm = row_tile_max(s_taddr, wb);
        if (m == -INFINITY) m = tm;
      }
      // P buffer par is free (and O_par stable) once P.V of tile j-2 finished
      if (!(ok = mbar_wait_warp(&sh->p_empty[par], ph ^ 1, a.err, abort))) break;
      bool over;
      float lt = row_exp_pass(s_taddr, wb, c, m, pb, i, over);
      if (__any_sync(0xFFFFFFFFu, over)) {
        const RowState rs =
            row_rescale_redo(s_taddr, o_taddr, wb[0], wb[1], wb[2], wb[3], c, m, l, over, j, pb, i);
        m = rs.m;
        l = rs.l;
        lt = rs.lt;
      }
      l += lt;
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sh->s_empty[par]);  // S_j consumed
        mbar_arrive(&sh->p_full[par]);   // P_j ready
      }
    }

    // epilogue: merge the two parities, O / l (+ output gate), bf16 store of
    // this warp's 64 output channels (par * 64 ..)
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
      const uint32_t col0 = par * 64;
      __nv_bfloat16* orow =
          static_cast<__nv_bfloat16*>(a.out) + grow * a.out_stride + h * kAtD + col0;
      const __nv_bfloat16* grow_p =
          a.og ? static_cast<const __nv_bfloat16*>(a.og) + grow * a.og_stride + h * kAtD + col0
               : nullptr;
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
          const uint4* gp = reinterpret_cast<const uint4*>(grow_p + cc * 32);
#pragma unroll
          for (int qd = 0; qd < 4; ++qd) {
            const uint4 gv = gp[qd];
            const __nv_bfloat16* ge = reinterpret_cast<const __nv_bfloat16*>(&gv);
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
              const int idx = qd * 8 + e;
              const float o0 = bf16_round(__uint_as_float(ov[idx]));
              const float o1 = bf16_round(__uint_as_float(ov[idx + 1]));
              const float g0 = bf16_round(sigmoid_ref(__bfloat162float(ge[e])));
              const float g1 = bf16_round(sigmoid_ref(__bfloat162float(ge[e + 1])));
              packed[idx >> 1] = pack_bf16x2(o0 * g0, o1 * g1);
            }
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

cudaError_t launch_masked_attention(const CUtensorMap& qmap, const CUtensorMap& kmap,
                                    const CUtensorMap& vmap, const MaskedAttnArgs& a,
                                    cudaStream_t stream) {
  if (a.B == 0 || a.Tq == 0 || a.Tkv == 0) return cudaSuccess;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(masked_attn_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kAtSmemBytes);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const int n_qt = (a.Tq + kAtBM - 1) / kAtBM;
  dim3 grid(n_qt, a.H, a.B);
  masked_attn_kernel<<<grid, kAtThreads, kAtSmemBytes, stream>>>(qmap, kmap, vmap, a);
  return cudaGetLastError();
}

}  // namespace gsa
