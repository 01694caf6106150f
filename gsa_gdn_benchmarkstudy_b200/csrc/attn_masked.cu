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
//   warps 0-3  softmax + epilogue (thread = query row = TMEM lane)
//   warp 4     TMA producer (Q once; K and V 128x128 tiles, 2-stage rings)
//   warp 5     TMEM owner + single-thread tcgen05.mma issuer
// Two passes over the key tiles (exact, no running rescale):
//   pass 1: S = Q.K^T into one of two TMEM S buffers; softmax warps take the
//           row max over selected keys.
//   pass 2: S again; p = 2^((s - m) * scale * log2 e) for selected keys, 0
//           otherwise; row sum l in fp32; P (bf16) written to shared memory in
//           the 128B-swizzled K-major layout; O += P.V accumulates in TMEM.
// Epilogue: o = O / l, rounded to bf16; optional gate bf16(o * bf16(sigmoid(og))).
//
// TMEM: S0 [0,128), S1 [128,256), O [256,384) fp32 columns (512 allocated).
// Shared memory: Q 32 KB, K 2x32 KB, V 2x32 KB, P 32 KB (one CTA per SM).
#include "kernels.h"

namespace gsa {
namespace {

constexpr int kAtBM = 128;
constexpr int kAtBN = 128;
constexpr int kAtD = 128;
constexpr int kAtTileBytes = kAtBM * kAtD * 2;  // 32 KB: two 128x64 swizzled boxes
constexpr int kAtBoxBytes = kAtTileBytes / 2;   // 16 KB
constexpr int kAtThreads = 192;
constexpr int kAtTmemCols = 512;

struct AtSmem {
  uint64_t q_full;
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2], s_empty[2];
  uint64_t p_full, p_empty;
  uint64_t o_full;
  uint32_t tmem_base;
  int abort;
};
constexpr int kAtSmemBytes = 1024 + 6 * kAtTileBytes + 256;

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

__global__ void __launch_bounds__(kAtThreads, 1)
    masked_attn_kernel(const __grid_constant__ CUtensorMap qmap,
                       const __grid_constant__ CUtensorMap kmap,
                       const __grid_constant__ CUtensorMap vmap, MaskedAttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* q_s = smem;
  uint8_t* k_s = smem + kAtTileBytes;      // 2 stages
  uint8_t* v_s = smem + 3 * kAtTileBytes;  // 2 stages
  uint8_t* p_s = smem + 5 * kAtTileBytes;
  AtSmem* sh = reinterpret_cast<AtSmem*>(smem + 6 * kAtTileBytes);

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
    }
    mbar_init(&sh->p_full, 4);
    mbar_init(&sh->p_empty, 1);
    mbar_init(&sh->o_full, 1);
    sh->abort = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(&sh->tmem_base, kAtTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;
  volatile int* abort = &sh->abort;

  if (warp == 4) {
    // ---------------------------------------------------------- TMA producer
    if (lane == 0) {
      prefetch_tmap(&qmap);
      prefetch_tmap(&kmap);
      prefetch_tmap(&vmap);
      const int x0 = h * kAtD;
      mbar_arrive_expect_tx(&sh->q_full, kAtTileBytes);
      tma_load_3d(q_s, &qmap, x0, row0, b, &sh->q_full);
      tma_load_3d(q_s + kAtBoxBytes, &qmap, x0 + 64, row0, b, &sh->q_full);
      int kit = 0, vit = 0;
      bool ok = true;
      for (int pass = 0; pass < 2 && ok; ++pass) {
        for (int j = 0; j < nt; ++j) {
          {
            const int st = kit & 1;
            if (!mbar_wait(&sh->k_empty[st], ((kit >> 1) & 1) ^ 1, a.err, abort)) { ok = false; break; }
            uint8_t* dst = k_s + st * kAtTileBytes;
            mbar_arrive_expect_tx(&sh->k_full[st], kAtTileBytes);
            tma_load_3d(dst, &kmap, x0, j * kAtBN, b, &sh->k_full[st]);
            tma_load_3d(dst + kAtBoxBytes, &kmap, x0 + 64, j * kAtBN, b, &sh->k_full[st]);
            ++kit;
          }
          if (pass == 1) {
            const int st = vit & 1;
            if (!mbar_wait(&sh->v_empty[st], ((vit >> 1) & 1) ^ 1, a.err, abort)) { ok = false; break; }
            uint8_t* dst = v_s + st * kAtTileBytes;
            mbar_arrive_expect_tx(&sh->v_full[st], kAtTileBytes);
            tma_load_3d(dst, &vmap, x0, j * kAtBN, b, &sh->v_full[st]);
            tma_load_3d(dst + kAtBoxBytes, &vmap, x0 + 64, j * kAtBN, b, &sh->v_full[st]);
            ++vit;
          }
        }
      }
    }
  } else if (warp == 5) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(kAtBM, kAtBN, 0, 0);   // Q K-major, K K-major
      constexpr uint32_t idesc_o = idesc_bf16_f32(kAtBM, kAtD, 0, 1);    // P K-major, V MN-major
      const uint32_t q_base = smem_u32(q_s);
      const uint32_t k_base = smem_u32(k_s);
      const uint32_t v_base = smem_u32(v_s);
      const uint32_t p_base = smem_u32(p_s);
      int sit = 0, kit = 0, vit = 0;
      bool ok = mbar_wait(&sh->q_full, 0, a.err, abort);

      auto issue_s = [&]() -> bool {
        const int sb = sit & 1, st = kit & 1;
        if (!mbar_wait(&sh->k_full[st], (kit >> 1) & 1, a.err, abort)) return false;
        if (!mbar_wait(&sh->s_empty[sb], ((sit >> 1) & 1) ^ 1, a.err, abort)) return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kAtD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kAtBoxBytes + (kk & 3) * 32;
          const uint64_t ad = sdesc_sw128(q_base + off, 16, 1024);
          const uint64_t bd = sdesc_sw128(k_base + st * kAtTileBytes + off, 16, 1024);
          tc_mma_ss(tmem + sb * kAtBN, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
        tc_commit(&sh->s_full[sb]);
        tc_commit(&sh->k_empty[st]);
        ++sit;
        ++kit;
        return true;
      };

      // pass 1: scores only
      for (int j = 0; ok && j < nt; ++j) ok = issue_s();
      // pass 2: scores again, then O += P.V once the softmax warps wrote P
      if (ok) ok = issue_s();
      for (int j = 0; ok && j < nt; ++j) {
        if (j + 1 < nt) {
          ok = issue_s();
          if (!ok) break;
        }
        const int vst = vit & 1;
        if (!mbar_wait(&sh->v_full[vst], (vit >> 1) & 1, a.err, abort)) { ok = false; break; }
        if (!mbar_wait(&sh->p_full, j & 1, a.err, abort)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kAtBN / 16; ++kk) {
          const uint64_t ad =
              sdesc_sw128(p_base + (kk >> 2) * kAtBoxBytes + (kk & 3) * 32, 16, 1024);
          const uint64_t bd =
              sdesc_sw128(v_base + vst * kAtTileBytes + kk * 16 * 128, kAtBoxBytes, 1024);
          tc_mma_ss(tmem + 2 * kAtBN, ad, bd, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(&sh->p_empty);
        tc_commit(&sh->v_empty[vst]);
        ++vit;
      }
      if (ok) tc_commit(&sh->o_full);
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------- softmax warps
    const int i = tid;
    const int r = row0 + i;
    const bool row_ok = r < a.Tq;
    const int64_t grow = static_cast<int64_t>(b) * a.Tq + r;
    const uint32_t* bm = a.bitmask + grow * a.bitmask_words;
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    const float c = a.scale * 1.4426950408889634f;
    const uint32_t p_row = smem_u32(p_s);
    int sit = 0;
    bool ok = true;

    // pass 1: row max over selected keys (raw dot-product units)
    float m = -INFINITY;
    for (int j = 0; j < nt; ++j) {
      const int sb = sit & 1;
      uint4 bits = make_uint4(0, 0, 0, 0);
      if (row_ok) bits = *reinterpret_cast<const uint4*>(bm + j * 4);
      if (!mbar_wait_warp(&sh->s_full[sb], (sit >> 1) & 1, a.err, abort)) { ok = false; break; }
      tc_fence_after();
      const uint32_t wbits[4] = {bits.x, bits.y, bits.z, bits.w};
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t raw[32];
        tmem_ld32(tmem + lane_base + sb * kAtBN + cc * 32, raw);
        tc_wait_ld();
        const uint32_t wb = wbits[cc];
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if ((wb >> e) & 1u) m = fmaxf(m, __uint_as_float(raw[e]));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->s_empty[sb]);
      ++sit;
    }
    if (m == -INFINITY) m = 0.f;
    const float mc = m * c;

    // pass 2: probabilities, P tile, row sum
    float l = 0.f;
    for (int j = 0; ok && j < nt; ++j) {
      const int sb = sit & 1;
      uint4 bits = make_uint4(0, 0, 0, 0);
      if (row_ok) bits = *reinterpret_cast<const uint4*>(bm + j * 4);
      if (!mbar_wait_warp(&sh->s_full[sb], (sit >> 1) & 1, a.err, abort)) { ok = false; break; }
      tc_fence_after();
      // P of the previous tile must have been consumed by its P.V MMA.
      if (!mbar_wait_warp(&sh->p_empty, (j & 1) ^ 1, a.err, abort)) { ok = false; break; }
      const uint32_t wbits[4] = {bits.x, bits.y, bits.z, bits.w};
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t raw[32];
        tmem_ld32(tmem + lane_base + sb * kAtBN + cc * 32, raw);
        tc_wait_ld();
        const uint32_t wb = wbits[cc];
        uint32_t packed[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float p0 = 0.f, p1 = 0.f;
          if ((wb >> e) & 1u) p0 = fast_ex2(fmaf(__uint_as_float(raw[e]), c, -mc));
          if ((wb >> (e + 1)) & 1u) p1 = fast_ex2(fmaf(__uint_as_float(raw[e + 1]), c, -mc));
          l += p0;
          l += p1;
          packed[e >> 1] = pack_bf16x2(p0, p1);
        }
        // keys 32cc..32cc+31 -> box cc/2, 16-byte chunks 4*(cc%2) .. +3 of row i
        const uint32_t box = p_row + (cc >> 1) * kAtBoxBytes;
#pragma unroll
        for (int qd = 0; qd < 4; ++qd) {
          const uint32_t chunk = (cc & 1) * 4 + qd;
          st_shared_v4(box + sw128_offset(i, chunk), packed[4 * qd], packed[4 * qd + 1],
                       packed[4 * qd + 2], packed[4 * qd + 3]);
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sh->s_empty[sb]);
        mbar_arrive(&sh->p_full);
      }
      ++sit;
    }

    // epilogue: O / l (+ output gate), bf16 store
    if (ok && mbar_wait_warp(&sh->o_full, 0, a.err, abort)) {
      tc_fence_after();
      const float inv_l = l > 0.f ? 1.0f / l : 0.f;
      __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(a.out) + grow * a.out_stride + h * kAtD;
      const __nv_bfloat16* grow_p =
          a.og ? static_cast<const __nv_bfloat16*>(a.og) + grow * a.og_stride + h * kAtD : nullptr;
#pragma unroll
      for (int cc = 0; cc < kAtD / 32; ++cc) {
        uint32_t raw[32];
        tmem_ld32(tmem + lane_base + 2 * kAtBN + cc * 32, raw);
        tc_wait_ld();
        if (!row_ok) continue;
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
              const float o0 = bf16_round(__uint_as_float(raw[idx]) * inv_l);
              const float o1 = bf16_round(__uint_as_float(raw[idx + 1]) * inv_l);
              const float g0 = bf16_round(sigmoid_ref(__bfloat162float(ge[e])));
              const float g1 = bf16_round(sigmoid_ref(__bfloat162float(ge[e + 1])));
              packed[idx >> 1] = pack_bf16x2(o0 * g0, o1 * g1);
            }
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; e += 2)
            packed[e >> 1] = pack_bf16x2(__uint_as_float(raw[e]) * inv_l,
                                         __uint_as_float(raw[e + 1]) * inv_l);
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
  if (warp == 5) {
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
