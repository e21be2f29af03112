// Per-chunk gradients of the backward on the 5th-generation tensor cores,
// sm_100a: bf16 inputs, dk = dv = 128, dense rows or packed sequences (exact
// semantics).  Replaces the warp-level bwd_grads_kernel (chunk_bwd.cu) at
// these shapes.  It is the last step of the reverse-mode differentiation of
// the chunk path (ops.py:299-346, the reference's jax.grad target): with the
// state h entering the chunk, the gradient dh of the state leaving it, V' and
// dX (all from the workspace the earlier launches filled), per chunk of C = 64
// tokens and value head (e = e^G, d = e^{G_C - G}, E_ij = e^{G_i - G_j}):
//
//   dAE = -tril_{-1}(dX V'^T) o E          dPE = tril_0(dO V'^T) o E
//   dQ  = e (dO h^T) + dPE K
//   dK  = d (V' dh^T) - beta e (dX h^T) + dPE^T Q + beta (dAE K) + dAE^T (beta K)
//   dV  = beta dX
//   dbeta = rowsum(dX o V) - e rowsum(K o dX h^T) + rowsum(dAE o K K^T)
//   dG  = -d rowsum(K o V' dh^T) + e rowsum(Q o dO h^T) - beta e rowsum(K o dX h^T)
//         + rowsum - colsum of (dPE o Q K^T + dAE o beta K K^T)
//   dG_C += e^{G_C} <h, dh> + sum(d K o V' dh^T);   dg = reverse in-chunk cumsum of dG.
//
// Persistent, one CTA per SM, one (chunk, head) item at a time.  Warp 0 loads
// q, k and dO by TMA and issues the products; warp 1 forms the gate vectors one
// item ahead; eight warps convert dX, V', h, dh to bf16 tiles and run the
// epilogues.  After the tcgen05 scans (dense rows), those four arrive as bf16
// (the hand-off) and warp 0 loads them with the item's q, k, dO, one item ahead.  Products (tcgen05.mma kind::f16, M = 128, fp32 in TMEM), stacked
// so that everything dK needs sits on TMEM lanes 0-63 and everything dQ needs
// on lanes 64-127:
//   P1 = [dX; dO] V'^T     P2 = [K; Q] K^T          (64 columns each)
//   P3 = [dX; dO] h^T      P4 = [V'; -] dh^T        (128 columns each)
//   P5 = [dAE; dPE] K      P6 = [dPE^T | dAE^T] [Q; beta K]
// Operands are bf16 (dX, V', h, dh, dPE, dAE rounded once); accumulation and
// every elementwise step are fp32.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "chunk_common.cuh"
#include "gdn_common.cuh"
#include "gdn_internal.h"
#include "ptx.cuh"

namespace gdn {

namespace {

constexpr int GR_D = 128;            // dk = dv
constexpr int kGrThreads = 320;

// Shared memory from a 1024-byte aligned base; every tile is bf16, rows of
// 128 bytes, 128-byte swizzled, in 64-column blocks.
struct GrLay {
  static constexpr int SM_KQ = 0;          // [kb][K 8 KB | Q 8 KB], kb = 0, 1      (TMA)
  static constexpr int SM_XO = 32768;      // [cb][dX 8 KB | dO 8 KB]               (dO by TMA)
  static constexpr int SM_VP = 65536;      // [cb][V' 8 KB]
  static constexpr int SM_H = 81920;       // [cb][h: 128 key rows, 16 KB]
  static constexpr int SM_DH = 114688;     // [cb][dh: 128 key rows, 16 KB]
  static constexpr int SM_AP = 147456;     // [dAE rows 0-63 | dPE rows 64-127], 16 KB
  static constexpr int SM_QST = 163840;    // [kb][dQ rows 8 KB]: staging of its tensor stores
  static constexpr int SM_VEC = 180224;    // 2 x GrVec
  static constexpr int SM_RED = SM_VEC + 2 * 1536;   // per-token partial sums
  static constexpr int SM_BAR = SM_RED + 24 * 64 * 4;
  static constexpr int SM_TMEM = SM_BAR + 16 * 8;
  static constexpr int SMEM_BYTES = SM_TMEM + 16 + 1024;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
};

// Gate vectors of one chunk.
struct GrVec {
  float G[C], e[C], d[C], beta[C], be[C];
  float eGC;
  float pad[63];
};
static_assert(sizeof(GrVec) == 1536, "gate vector size");

// Per-token partial sums in SM_RED (64 floats each), each written by one
// thread and summed in a fixed order (no atomics: the gradients are the same
// on every run).
enum {
  RD_G = 0,       // [4] dG from the first epilogue: row sums by side (dAE, dPE) x column half
  RD_C = 4,       // [4] its column sums, by TMEM lane quarter (subtracted)
  RD_B = 8,       // [2] dbeta: rowsum(dAE o K K^T), by column half
  RD_XV = 10,     // dbeta: rowsum(dX o V)
  RD_KG = 11,     // [2] dG from the dK side of the last epilogue, by column half
  RD_KB = 13,     // [2] dbeta from the dK side
  RD_KC = 15,     // [2] d rowsum(K o V' dh^T), for dG_C
  RD_QG = 17,     // [2] dG from the dQ side
  RD_HD = 19,     // <h, dh> partials of the eight math warps
  RD_N = 20,
  RD_XVP = 20,    // [4] (hand-off) rowsum(dX o v) by 32-column block, [64 tokens][4], loaded
};

enum {
  G_FULL = 0,     // q, k, dO of the item landed
  G_VFULL = 1,    // [2] gate vectors ready
  G_VEMPTY = 3,   // [2] gate vectors read
  G_CONV = 5,     // bf16 tiles written (dX, V', h, dh, beta K)
  G_M12 = 6,      // P1, P2 in TMEM
  G_AP = 7,       // dAE / dPE tile written
  G_M3456 = 8,    // P3 .. P6 in TMEM: every product of the item complete
  G_KQFREE = 9,   // the last epilogue's reads of K, Q and of P3 .. P6 done (8 warps)
  G_FULL2 = 10,   // dO (and the hand-off's V', dX, h, dh, rowsum partials) landed
  G_HFREE = 11,   // (hand-off) h, dh and the rowsum partials read (8 warps)
  G_M1234 = 12,   // P1 .. P4 complete: dO, V', dX, h, dh no longer read
};

// TMEM columns (the CTA has the SM to itself)
constexpr uint32_t GT_P1 = 0, GT_P2 = 64, GT_P5 = 0, GT_P3 = 128, GT_P4 = 256, GT_P6 = 384,
                   GT_COLS = 512;

constexpr uint32_t IDESC_N64_KK = idesc_bf16(128, 64, 0, 0);
constexpr uint32_t IDESC_N128_KK = idesc_bf16(128, 128, 0, 0);
constexpr uint32_t IDESC_N128_KM = idesc_bf16(128, 128, 0, 1);
constexpr uint32_t IDESC_N128_MM = idesc_bf16(128, 128, 1, 1);

// After the call, lane l holds the sum over the warp's 32 lanes of v[l]
// (a butterfly reduce-scatter: 31 shuffles instead of 32 x 5).
__device__ __forceinline__ float warp_colsum32(float (&v)[32], int lane) {
#pragma unroll
  for (int w = 16; w >= 1; w >>= 1) {
    const bool up = (lane & w) != 0;
#pragma unroll
    for (int c = 0; c < w; ++c) {
      const float send = up ? v[c] : v[c + w];
      const float keep = up ? v[c + w] : v[c];
      v[c] = keep + __shfl_xor_sync(0xffffffffu, send, w);
    }
  }
  return v[0];
}

__global__ void __launch_bounds__(kGrThreads, 1)
bwd_grads_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmQ,
                    const __grid_constant__ CUtensorMap tmO, const __nv_bfloat16* __restrict__ v,
                    const float* __restrict__ g, const float* __restrict__ beta,
                    const float* __restrict__ UV, const float* __restrict__ YX,
                    const float* __restrict__ hs, const float* __restrict__ dhs,
                    __nv_bfloat16* __restrict__ dq, __nv_bfloat16* __restrict__ dk,
                    __nv_bfloat16* __restrict__ dvo, float* __restrict__ dg,
                    float* __restrict__ dbeta, float* __restrict__ dqk,
                    const int* __restrict__ cu, const int* __restrict__ coff, int n_seqs, int B,
                    int T, int H, int Hk, int N, const unsigned char* __restrict__ hb,
                    const unsigned char* __restrict__ dhb,
                    const __grid_constant__ CUtensorMap tmVP,
                    const __grid_constant__ CUtensorMap tmDX,
                    const __grid_constant__ CUtensorMap tmDQ,
                    const __grid_constant__ CUtensorMap tmDK, int tma_out) {
  // tma_out (dense rows, dq and dk written directly): each item's dK and dQ
  // rows are staged as bf16 tiles (dK over the dAE / dPE tile, which P5 and P6
  // no longer read, dQ in SM_QST) and written by four tensor stores, instead
  // of 16-byte stores scattered over 64 rows 4 KB apart
  // hb / dhb (the scans' hand-off; dense rows only): h and dh of every (chunk,
  // head) as the bf16 tiles the scan kernels wrote (32 and 36 KB slots, [column
  // tile][128 key rows][128 B], 128-byte swizzled), loaded by bulk copies with
  // the rowsum(dX o v) partials (each dhs slot + 32 KB); V' and dX loaded by
  // TMA (tmVP, tmDX: bf16 rows [slots C][dv], 64 x 64 boxes, 128-byte swizzle).
  // Nothing is converted and dV is not formed here (the reverse scan wrote it).
  using L = GrLay;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  unsigned char* sm = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::SM_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + L::SM_TMEM);
  GrVec* vecs = reinterpret_cast<GrVec*>(sm + L::SM_VEC);
  float* red = reinterpret_cast<float*>(sm + L::SM_RED);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Items w = blockIdx.x + j gridDim.x: value head h = w % H of global chunk
  // gc = w / H (workspace rows (gc H + h) C ..).  Dense: chunk n of row b is
  // gc = b N + n.  Packed (n_seqs > 0): one row of T tokens, sequence s owns
  // the chunks coff[s] .. coff[s + 1] - 1.
  const long long total = (long long)(n_seqs ? coff[n_seqs] : B * N) * H;
  const int cnt = blockIdx.x < total ? (int)((total - 1 - blockIdx.x) / gridDim.x) + 1 : 0;
  struct Item {
    int gc, h, hq, b, tok, len;   // tok: first token of the chunk in row b; len: its tokens
  };
  // (32-bit division where the item count allows: the 64-bit one is a long
  // software sequence, and every warp decodes every item)
  const bool small = total < (1LL << 31);
  auto item = [&](int j) {
    const long long w = blockIdx.x + (long long)j * gridDim.x;
    Item it;
    if (small) {
      const unsigned w32 = (unsigned)w;
      it.gc = (int)(w32 / (unsigned)H);
      it.h = (int)(w32 - (unsigned)it.gc * (unsigned)H);
    } else {
      it.h = (int)(w % H);
      it.gc = (int)(w / H);
    }
    it.hq = it.h * Hk / H;
    if (!n_seqs) {
      it.b = it.gc / N;
      it.tok = (it.gc - it.b * N) * C;
      it.len = min(C, T - it.tok);
    } else {
      int lo = 0, hi = n_seqs;   // coff[lo] <= gc < coff[hi]
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (coff[mid] <= it.gc) lo = mid; else hi = mid;
      }
      const int a0 = min(max(cu[lo], 0), T);
      const int a1 = min(max(cu[lo + 1], a0), T);
      it.b = 0;
      it.tok = a0 + (it.gc - coff[lo]) * C;
      it.len = min(C, a1 - it.tok);
    }
    return it;
  };

  if (tid == 0) {
    mbar_init(&bars[G_FULL], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[G_VFULL + i], 1);
      mbar_init(&bars[G_VEMPTY + i], 1);
    }
    mbar_init(&bars[G_CONV], 8);
    mbar_init(&bars[G_M12], 1);
    mbar_init(&bars[G_AP], 8);
    mbar_init(&bars[G_M3456], 1);
    mbar_init(&bars[G_KQFREE], 8);
    mbar_init(&bars[G_FULL2], 1);
    mbar_init(&bars[G_HFREE], 8);
    mbar_init(&bars[G_M1234], 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, GT_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sbase = smem_u32(sm);

  if (warp == 0) {
    // ---- loads (TMA, bulk copies) and the products ----
    if (lane == 0 && cnt > 0) {
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmO);
      // G_FULL2: everything the products P1 .. P4 read (dO; with the hand-off
      // also V', dX, h, dh and the rowsum partials), loaded once P1 .. P4 of
      // the previous item completed (its epilogues still running); G_FULL: K
      // and Q, which P5, P6 and the last epilogue also read, loaded once those
      // have
      auto load_a = [&](int j) {
        const Item it = item(j);
        mbar_arrive_expect_tx(&bars[G_FULL2], hb ? 16384 + 65536 + 32768 + 1024 : 16384);
        if (hb) {
          const size_t ws = (size_t)it.gc * H + it.h;
          bulk_g2s(sm + L::SM_H, hb + ws * kHandoffHSlot, 32768, &bars[G_FULL2]);
          bulk_g2s(sm + L::SM_DH, dhb + ws * kHandoffDhSlot, 32768, &bars[G_FULL2]);
          bulk_g2s(sm + L::SM_RED + RD_XVP * 256, dhb + ws * kHandoffDhSlot + 32768, 1024,
                   &bars[G_FULL2]);
          for (int cb = 0; cb < 2; ++cb) {
            tma_load_2d(sm + L::SM_VP + cb * 8192, &tmVP, 64 * cb, (int)(ws * C), &bars[G_FULL2]);
            tma_load_2d(sm + L::SM_XO + cb * 16384, &tmDX, 64 * cb, (int)(ws * C),
                        &bars[G_FULL2]);
          }
        }
        for (int kb = 0; kb < 2; ++kb)
          tma_load_4d(sm + L::SM_XO + kb * 16384 + 8192, &tmO, 64 * kb, it.h, it.tok, it.b,
                      &bars[G_FULL2]);
      };
      auto load_b = [&](int j) {
        const Item it = item(j);
        mbar_arrive_expect_tx(&bars[G_FULL], 32768);
        for (int kb = 0; kb < 2; ++kb) {
          tma_load_4d(sm + L::SM_KQ + kb * 16384, &tmK, 64 * kb, it.hq, it.tok, it.b, &bars[G_FULL]);
          tma_load_4d(sm + L::SM_KQ + kb * 16384 + 8192, &tmQ, 64 * kb, it.hq, it.tok, it.b,
                      &bars[G_FULL]);
        }
      };
      const uint32_t kq = sbase + L::SM_KQ, xo = sbase + L::SM_XO, vp = sbase + L::SM_VP;
      const uint32_t hh = sbase + L::SM_H, dh = sbase + L::SM_DH, ap = sbase + L::SM_AP;
      load_a(0);
      load_b(0);
      int pend_a = 0, pend_b = 0;   // items whose loads were issued and not yet seen (-1: none)
      for (int j = 0; j < cnt; ++j) {
        bool ok = mbar_wait(&bars[G_FULL2], (uint32_t)j & 1u) &&
                  mbar_wait(&bars[G_FULL], (uint32_t)j & 1u);
        pend_a = pend_b = -1;
        // with the hand-off, P1 .. P4 read only loaded tiles
        ok = ok && (hb || mbar_wait(&bars[G_CONV], (uint32_t)j & 1u));
        if (!ok) break;
        tc_fence_after();
        // P2 = [K;Q] K^T and P1 = [dX;dO] V'^T (K-dim 128 in 8 steps of 16)
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (k >> 2) * 16384 + (k & 3) * 32;
          mma_bf16(tmem + GT_P2, umma_desc(kq + off, 16, 1024, SW128),
                   umma_desc(kq + off, 16, 1024, SW128), IDESC_N64_KK, k > 0);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (k >> 2) * 16384 + (k & 3) * 32;
          mma_bf16(tmem + GT_P1, umma_desc(xo + off, 16, 1024, SW128),
                   umma_desc(vp + (k >> 2) * 8192 + (k & 3) * 32, 16, 1024, SW128), IDESC_N64_KK,
                   k > 0);
        }
        mma_commit(&bars[G_M12]);
        // P3 = [dX;dO] h^T, P4 = [V'; -] dh^T (N = 128 key rows of h, dh)
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (k >> 2) * 16384 + (k & 3) * 32;
          mma_bf16(tmem + GT_P3, umma_desc(xo + off, 16, 1024, SW128),
                   umma_desc(hh + off, 16, 1024, SW128), IDESC_N128_KK, k > 0);
          mma_bf16(tmem + GT_P4, umma_desc(vp + (k >> 2) * 8192 + (k & 3) * 32, 16, 1024, SW128),
                   umma_desc(dh + off, 16, 1024, SW128), IDESC_N128_KK, k > 0);
        }
        mma_commit(&bars[G_M1234]);
        if (j + 1 < cnt) {
          // P1 .. P4 have read dO, V', dX, h, dh (and the epilogues their h,
          // dh, partials): the next item's, while this item's epilogues run
          if (!mbar_wait(&bars[G_M1234], (uint32_t)j & 1u) ||
              (hb && !mbar_wait(&bars[G_HFREE], (uint32_t)j & 1u)))
            break;
          load_a(j + 1);
          pend_a = j + 1;
        }
        ok = mbar_wait(&bars[G_AP], (uint32_t)j & 1u);
        if (!ok) break;
        tc_fence_after();
        // P5 = [beta dAE; dPE] K: A K-major over the chunk's tokens; B = K,
        // MN-major (N = dk in two 64-wide blocks 16 KB apart)
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + GT_P5, umma_desc(ap + k * 32, 16, 1024, SW128),
                   umma_desc(kq + k * 2048, 16384, 1024, SW128), IDESC_N128_KM, k > 0);
        // P6 = dPE^T Q + (beta dAE)^T K: A = dPE^T / (beta dAE)^T read MN-major
        // from the rows of the tile (M = 64 tokens; the second M block, 8 KB
        // on, is not used: rows 64-127 of P6 are ignored)
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + GT_P6, umma_desc(ap + 8192 + k * 2048, 8192, 1024, SW128),
                   umma_desc(kq + 8192 + k * 2048, 16384, 1024, SW128), IDESC_N128_MM, k > 0);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + GT_P6, umma_desc(ap + k * 2048, 8192, 1024, SW128),
                   umma_desc(kq + k * 2048, 16384, 1024, SW128), IDESC_N128_MM, 1u);
        mma_commit(&bars[G_M3456]);
        if (j + 1 < cnt) {
          // every product and the last epilogue have read K and Q: the next item's
          if (!mbar_wait(&bars[G_M3456], (uint32_t)j & 1u) ||
              !mbar_wait(&bars[G_KQFREE], (uint32_t)j & 1u))
            break;
          load_b(j + 1);
          pend_b = j + 1;
        }
      }
      // (before the CTA exits)
      if (pend_a >= 0) mbar_wait(&bars[G_FULL2], (uint32_t)pend_a & 1u);
      if (pend_b >= 0) mbar_wait(&bars[G_FULL], (uint32_t)pend_b & 1u);
    }
  } else if (warp == 1) {
    // ---- gate vectors, one item ahead ----
    float g0 = 0.f, g1 = 0.f, b0 = 0.f, b1 = 0.f;
    auto fetch = [&](int j) {
      const Item it = item(j);
      const size_t gb = ((size_t)it.b * T + it.tok) * H + it.h;
      const int i = 2 * lane;
      g0 = i < it.len ? ldg_f32(g + gb + (size_t)i * H) : 0.f;
      g1 = i + 1 < it.len ? ldg_f32(g + gb + (size_t)(i + 1) * H) : 0.f;
      b0 = i < it.len ? ldg_f32(beta + gb + (size_t)i * H) : 0.f;
      b1 = i + 1 < it.len ? ldg_f32(beta + gb + (size_t)(i + 1) * H) : 0.f;
    };
    if (cnt > 0) fetch(0);
    for (int j = 0; j < cnt; ++j) {
      const int s = j & 1;
      if (j >= 2 && !mbar_wait(&bars[G_VEMPTY + s], (uint32_t)((j - 2) >> 1) & 1u)) break;
      GrVec& vb = vecs[s];
      const float pair = g0 + g1;
      float incl = pair;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += y;
      }
      const float G0 = incl - pair + g0, G1 = incl;
      const float GC = __shfl_sync(0xffffffffu, incl, 31);
      vb.G[2 * lane] = G0;
      vb.G[2 * lane + 1] = G1;
      vb.e[2 * lane] = gate_exp(G0);
      vb.e[2 * lane + 1] = gate_exp(G1);
      vb.d[2 * lane] = gate_exp(GC - G0);
      vb.d[2 * lane + 1] = gate_exp(GC - G1);
      vb.beta[2 * lane] = b0;
      vb.beta[2 * lane + 1] = b1;
      vb.be[2 * lane] = b0 * gate_exp(G0);
      vb.be[2 * lane + 1] = b1 * gate_exp(G1);
      if (lane == 0) vb.eGC = gate_exp(GC);
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[G_VFULL + s]);
      if (j + 1 < cnt) fetch(j + 1);
    }
  } else {
    // ---- the math warps ----
    const int pw = warp - 2;          // 0..7
    const int pi = tid - 64;          // 0..255
    const int wq = warp & 3;          // TMEM lane quarter this warp may read
    const int ch = pw >> 2;           // which half of the accumulator columns
    const int p = wq * 32 + lane;     // TMEM lane
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    const size_t plane = (size_t)B * T * H * GR_D;   // per value head dq / dk planes (grouped)
    bool ok = true;
    for (int j = 0; j < cnt; ++j) {
      const int s = j & 1;
      const Item it = item(j);
      const size_t slot = (size_t)it.gc * H + it.h;   // workspace slot of (chunk, head)
      const GrVec& vb = vecs[s];
      ok = mbar_wait(&bars[G_VFULL + s], (uint32_t)(j >> 1) & 1u) && ok;

      // ---- without the hand-off: bf16 tiles of dX (over the [dX; dO]
      //      blocks), V', h, dh; dV = beta dX; rowsum(dX o V); <h, dh> ----
      if (!hb) {
        const int m = pi >> 2, c0 = (pi & 3) * 32, cb = c0 >> 6, k8 = (c0 & 63) >> 3;
        const bool valid = m < it.len;
        const size_t trow = ((size_t)it.b * T + it.tok + m) * H + it.h;   // token row (valid)
        const float* xr = YX + (slot * C + m) * GR_D + c0;
        const float* vr = UV + (slot * C + m) * GR_D + c0;
        float x[32], w[32];
#pragma unroll
        for (int c = 0; c < 32; c += 4) {
          const float4 a4 = *reinterpret_cast<const float4*>(xr + c);
          const float4 b4 = *reinterpret_cast<const float4*>(vr + c);
          x[c] = a4.x; x[c + 1] = a4.y; x[c + 2] = a4.z; x[c + 3] = a4.w;
          w[c] = b4.x; w[c + 1] = b4.y; w[c + 2] = b4.z; w[c + 3] = b4.w;
        }
        float xv = 0.f;
        if (valid) {
          const __nv_bfloat16* vin = v + trow * GR_D + c0;
          const float bm = vb.beta[m];
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            float vv[8], o8[8];
            unpack_bf16x8(*reinterpret_cast<const uint4*>(vin + 8 * c8), vv);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              xv = fmaf(x[8 * c8 + e], vv[e], xv);
              o8[e] = bm * x[8 * c8 + e];
            }
            *reinterpret_cast<uint4*>(dvo + trow * GR_D + c0 + 8 * c8) = pack_bf16x8(o8);
          }
        }
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          *reinterpret_cast<uint4*>(sm + L::SM_XO + cb * 16384 + sw128(m, k8 + c8)) =
              pack_bf16x8(x + 8 * c8);
          *reinterpret_cast<uint4*>(sm + L::SM_VP + cb * 8192 + sw128(m, k8 + c8)) =
              pack_bf16x8(w + 8 * c8);
        }
        xv += __shfl_xor_sync(0xffffffffu, xv, 1);
        xv += __shfl_xor_sync(0xffffffffu, xv, 2);
        if ((pi & 3) == 0) red[RD_XV * 64 + m] = xv;
      }
      if (!hb) {
        // h and dh: key row r, 64 columns of block cb, in two halves of 32
        const int r = pi >> 1, cb = pi & 1;
        const float* hr = hs + (slot * GR_D + r) * GR_D + cb * 64;
        const float* dr = dhs + (slot * GR_D + r) * GR_D + cb * 64;
        float hd = 0.f;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          float a[32], d[32];
#pragma unroll
          for (int c = 0; c < 32; c += 4) {
            const float4 a4 = *reinterpret_cast<const float4*>(hr + 32 * half + c);
            const float4 d4 = *reinterpret_cast<const float4*>(dr + 32 * half + c);
            a[c] = a4.x; a[c + 1] = a4.y; a[c + 2] = a4.z; a[c + 3] = a4.w;
            d[c] = d4.x; d[c + 1] = d4.y; d[c + 2] = d4.z; d[c + 3] = d4.w;
          }
#pragma unroll
          for (int c = 0; c < 32; ++c) hd = fmaf(a[c], d[c], hd);
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            *reinterpret_cast<uint4*>(sm + L::SM_H + cb * 16384 + sw128(r, 4 * half + c8)) =
                pack_bf16x8(a + 8 * c8);
            *reinterpret_cast<uint4*>(sm + L::SM_DH + cb * 16384 + sw128(r, 4 * half + c8)) =
                pack_bf16x8(d + 8 * c8);
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) hd += __shfl_xor_sync(0xffffffffu, hd, o);
        if (lane == 0) red[RD_HD * 64 + pw] = hd;
      }
      if (!hb) {
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[G_CONV]);
        // the next item's rows of dX, V', v, h, dh into L2 (this thread's own
        // conversion reads), so that its conversion does not wait on DRAM
        if (j + 1 < cnt) {
          const Item nx = item(j + 1);
          const size_t ns = (size_t)nx.gc * H + nx.h;
          const int m = pi >> 2, c0 = (pi & 3) * 32, r = pi >> 1, cb = pi & 1;
          prefetch_l2(YX + (ns * C + m) * GR_D + c0);
          prefetch_l2(UV + (ns * C + m) * GR_D + c0);
          if (m < nx.len)
            prefetch_l2(v + (((size_t)nx.b * T + nx.tok + m) * H + nx.h) * GR_D + c0);
          const float* hr = hs + (ns * GR_D + r) * GR_D + cb * 64;
          const float* dr = dhs + (ns * GR_D + r) * GR_D + cb * 64;
          prefetch_l2(hr);
          prefetch_l2(hr + 32);
          prefetch_l2(dr);
          prefetch_l2(dr + 32);
        }
      }

      if (hb) {
        // ---- while P1, P2 run: <h, dh> from the bf16 tiles (key row pi / 2,
        //      column tile pi % 2) and the sum of the rowsum(dX o v) partials ----
        ok = mbar_wait(&bars[G_FULL2], (uint32_t)j & 1u) && ok;
        const int r = pi >> 1, cb = pi & 1;
        float hd = 0.f;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          float a8[8], d8[8];
          unpack_bf16x8(*reinterpret_cast<const uint4*>(sm + L::SM_H + cb * 16384 + sw128(r, c8)),
                        a8);
          unpack_bf16x8(*reinterpret_cast<const uint4*>(sm + L::SM_DH + cb * 16384 + sw128(r, c8)),
                        d8);
#pragma unroll
          for (int e = 0; e < 8; ++e) hd = fmaf(a8[e], d8[e], hd);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) hd += __shfl_xor_sync(0xffffffffu, hd, o);
        if (lane == 0) red[RD_HD * 64 + pw] = hd;
        if (pi < 64) {
          const float* xp = red + RD_XVP * 64 + pi * 4;
          red[RD_XV * 64 + pi] = (xp[0] + xp[1]) + (xp[2] + xp[3]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[G_HFREE]);
      }

      // ---- first epilogue: dAE (lanes 0-63) and dPE (lanes 64-127), row i,
      //      columns 32 ch ..; their row and column sums against K K^T / Q K^T ----
      ok = mbar_wait(&bars[G_M12], (uint32_t)j & 1u) && ok;
      tc_fence_after();
      {
        const int side = p >> 6, i = p & 63;
        float a[32], kk[32], col[32];
        tmem_ld32(tmem + GT_P1 + (uint32_t)ch * 32 + lane_off, a);
        tmem_ld32(tmem + GT_P2 + (uint32_t)ch * 32 + lane_off, kk);
        const bool row_in = i < it.len;
        const float Gi = vb.G[i], bi = vb.beta[i];
        float rg = 0.f, rb = 0.f;
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int jj = 32 * ch + e;
          const bool in = row_in && (side ? jj <= i : jj < i);
          const float E = in ? gate_exp(Gi - vb.G[jj]) : 0.f;
          // dAE = -(dX V'^T) E ; dPE = (dO V'^T) E
          const float val = side ? a[e] * E : -a[e] * E;
          const float xx = side ? val * kk[e] : val * bi * kk[e];
          if (!side) rb = fmaf(val, kk[e], rb);
          rg += xx;
          col[e] = xx;
          a[e] = side ? val : val * bi;   // the tile holds beta dAE
        }
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8)
          *reinterpret_cast<uint4*>(sm + L::SM_AP + sw128(p, 4 * ch + c8)) = pack_bf16x8(a + 8 * c8);
        red[(RD_G + 2 * side + ch) * 64 + i] = rg;
        if (!side) red[(RD_B + ch) * 64 + i] = rb;
        const float cs = warp_colsum32(col, lane);
        red[(RD_C + wq) * 64 + 32 * ch + lane] = cs;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[G_AP]);


      // ---- last epilogue: dK on lanes 0-63, dQ on lanes 64-127, token row m,
      //      key columns 64 ch .. 64 ch + 63 in four steps of 16 ----
      ok = mbar_wait(&bars[G_M3456], (uint32_t)j & 1u) && ok;
      ok = mbar_wait(&bars[G_FULL], (uint32_t)j & 1u) && ok;   // (K, Q rows read below)
      tc_fence_after();
      {
        const int side = p >> 6, m = p & 63;
        const bool valid = m < it.len;
        const size_t trow = ((size_t)it.b * T + it.tok + m);
        const float em = vb.e[m], dm = vb.d[m], bem = vb.be[m];
        float r1 = 0.f, r2 = 0.f;   // dK side: rowsum(K o Kd), rowsum(K o M); dQ side: rowsum(Q o Q0)
#pragma unroll 1
        for (int sub = 0; sub < 4; ++sub) {
          const int c = 64 * ch + 16 * sub, kb = c >> 6, k8 = (c & 63) >> 3;
          // this row's 16 key (side 0) or query (side 1) values, bf16 from shared memory
          float kr[16];
          const unsigned char* src = sm + L::SM_KQ + kb * 16384 + (side ? 8192 : 0);
          unpack_bf16x8(*reinterpret_cast<const uint4*>(src + sw128(m, k8)), kr);
          unpack_bf16x8(*reinterpret_cast<const uint4*>(src + sw128(m, k8 + 1)), kr + 8);
          float out[16];
          if (!side) {
            float Mv[16], Kd[16], AK[16], ak[16];
            tmem_ld16(tmem + GT_P3 + (uint32_t)c + lane_off, Mv);
            tmem_ld16(tmem + GT_P4 + (uint32_t)c + lane_off, Kd);
            tmem_ld16(tmem + GT_P5 + (uint32_t)c + lane_off, AK);
            tmem_ld16(tmem + GT_P6 + (uint32_t)c + lane_off, ak);
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              out[e] = dm * Kd[e] - bem * Mv[e] + ak[e] + AK[e];
              r1 = fmaf(kr[e], Kd[e], r1);
              r2 = fmaf(kr[e], Mv[e], r2);
            }
          } else {
            float Q0[16], PK[16];
            tmem_ld16(tmem + GT_P3 + (uint32_t)c + lane_off, Q0);
            tmem_ld16(tmem + GT_P5 + (uint32_t)c + lane_off, PK);
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              out[e] = fmaf(em, Q0[e], PK[e]);
              r1 = fmaf(kr[e], Q0[e], r1);
            }
          }
          if (tma_out) {
            // staged for the item's tensor stores (rows past the end of T are
            // clipped by the store): dK over the dAE / dPE tile, dQ in SM_QST
            unsigned char* stg = sm + (side ? L::SM_QST : L::SM_AP) + kb * 8192;
            *reinterpret_cast<uint4*>(stg + sw128(m, k8)) = pack_bf16x8(out);
            *reinterpret_cast<uint4*>(stg + sw128(m, k8 + 1)) = pack_bf16x8(out + 8);
          } else if (valid) {
            if (dqk) {   // grouped q/k heads: per value head, summed afterwards
              float* dst = dqk + (side ? 0 : plane) + (trow * H + it.h) * GR_D + c;
#pragma unroll
              for (int e = 0; e < 16; e += 4)
                *reinterpret_cast<float4*>(dst + e) =
                    make_float4(out[e], out[e + 1], out[e + 2], out[e + 3]);
            } else {
              __nv_bfloat16* dst = (side ? dq : dk) + (trow * Hk + it.hq) * GR_D + c;
              *reinterpret_cast<uint4*>(dst) = pack_bf16x8(out);
              *reinterpret_cast<uint4*>(dst + 8) = pack_bf16x8(out + 8);
            }
          }
        }
        // (the reads of K, Q and of the TMEM that the next item's products
        // overwrite are done)
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[G_KQFREE]);
        if (!side) {
          red[(RD_KG + ch) * 64 + m] = -dm * r1 - bem * r2;
          red[(RD_KB + ch) * 64 + m] = -em * r2;
          red[(RD_KC + ch) * 64 + m] = valid ? dm * r1 : 0.f;
        } else {
          red[(RD_QG + ch) * 64 + m] = em * r1;
        }
      }
      if (tma_out) fence_proxy_async_smem();
      tc_fence_before();
      named_sync(1, 256);
      if (tma_out && pi == 32) {
        // the item's dK and dQ rows: four tensor stores of 64 x 64 tiles
        for (int kb = 0; kb < 2; ++kb) {
          tma_store_4d(&tmDK, 64 * kb, it.hq, it.tok, it.b, sm + L::SM_AP + kb * 8192);
          tma_store_4d(&tmDQ, 64 * kb, it.hq, it.tok, it.b, sm + L::SM_QST + kb * 8192);
        }
        bulk_commit();
      }
      // ---- per token: dG, dbeta; dG_C; dg = reverse in-chunk cumsum of dG ----
      if (pi < 32) {
        const int l = pi;
        auto dG = [&](int m) {
          float x = (red[(RD_G + 0) * 64 + m] + red[(RD_G + 1) * 64 + m]) +
                    (red[(RD_G + 2) * 64 + m] + red[(RD_G + 3) * 64 + m]);
          x -= (red[(RD_C + 0) * 64 + m] + red[(RD_C + 1) * 64 + m]) +
               (red[(RD_C + 2) * 64 + m] + red[(RD_C + 3) * 64 + m]);
          x += (red[(RD_KG + 0) * 64 + m] + red[(RD_KG + 1) * 64 + m]) +
               (red[(RD_QG + 0) * 64 + m] + red[(RD_QG + 1) * 64 + m]);
          return m < it.len ? x : 0.f;
        };
        auto dB = [&](int m) {
          const float x = red[RD_XV * 64 + m] + (red[(RD_B + 0) * 64 + m] + red[(RD_B + 1) * 64 + m]) +
                          (red[(RD_KB + 0) * 64 + m] + red[(RD_KB + 1) * 64 + m]);
          return m < it.len ? x : 0.f;
        };
        // dG_C = e^{G_C} <h, dh> + sum over the chunk's tokens of d rowsum(K o V' dh^T)
        float hd = l < 8 ? red[RD_HD * 64 + l] : 0.f;
        float kc = (red[(RD_KC + 0) * 64 + l] + red[(RD_KC + 1) * 64 + l]) +
                   (red[(RD_KC + 0) * 64 + l + 32] + red[(RD_KC + 1) * 64 + l + 32]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          hd += __shfl_xor_sync(0xffffffffu, hd, o);
          kc += __shfl_xor_sync(0xffffffffu, kc, o);
        }
        const float y = fmaf(vb.eGC, hd, kc);
        float x0 = dG(l), x1 = dG(l + 32) + (l == 31 ? y : 0.f);
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y0 = __shfl_down_sync(0xffffffffu, x0, o);
          const float y1 = __shfl_down_sync(0xffffffffu, x1, o);
          if (l + o < 32) { x0 += y0; x1 += y1; }
        }
        x0 += __shfl_sync(0xffffffffu, x1, 0);
        const size_t t0 = ((size_t)it.b * T + it.tok) * H + it.h;
        if (l < it.len) {
          dg[t0 + (size_t)l * H] = x0;
          dbeta[t0 + (size_t)l * H] = dB(l);
        }
        if (l + 32 < it.len) {
          dg[t0 + (size_t)(l + 32) * H] = x1;
          dbeta[t0 + (size_t)(l + 32) * H] = dB(l + 32);
        }
        if (l == 0) mbar_arrive(&bars[G_VEMPTY + s]);
      }
      // the partial sums are read, and the stores have read their staging:
      // the next item may overwrite both
      if (tma_out && pi == 32) bulk_wait_read<0>();
      if (!named_sync_and(1, 256, ok)) break;
    }
    if (tma_out && pi == 32) bulk_wait<0>();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, GT_COLS);
  }
}

}  // namespace

GDN_DEVICE_ERROR_ACCESSOR(device_error_bwd_grads)

bool bwd_grads_tc_supported(int dtype, int dk, int dv) {
  return dtype == kBF16 && dk == GR_D && dv == GR_D && encode_fn() != nullptr;
}

cudaError_t launch_bwd_grads_tc(const BwdGradsArgs& a, cudaStream_t st) {
  const int rows = a.n_seqs ? 1 : a.B;
  if ((long long)rows * a.H == 0 || a.T == 0 || a.NC == 0) return cudaSuccess;
  const bool hand = a.hb != nullptr;
  if (hand && (a.n_seqs || !a.dhb || !a.vpb || !a.dxb)) return cudaErrorInvalidValue;
  const bool tma_out = !a.n_seqs && !a.dqk;
  CUtensorMap mk, mq, mo, mvp, mdx, mdq, mdk;
  const long long slot_rows = (long long)a.NC * a.H * C;
  if (!make_bf16_map_4d(&mk, a.k, rows, a.T, a.Hk, GR_D) ||
      !make_bf16_map_4d(&mq, a.q, rows, a.T, a.Hk, GR_D) ||
      !make_bf16_map_4d(&mo, a.dO, rows, a.T, a.H, GR_D) ||
      (hand && (!make_bf16_map_2d(&mvp, a.vpb, slot_rows, GR_D, true) ||
                !make_bf16_map_2d(&mdx, a.dxb, slot_rows, GR_D, true))) ||
      (tma_out && (!make_bf16_map_4d(&mdq, a.dq, rows, a.T, a.Hk, GR_D) ||
                   !make_bf16_map_4d(&mdk, a.dk, rows, a.T, a.Hk, GR_D))))
    return cudaErrorInvalidValue;
  if (!hand) mvp = mdx = mo;   // (not read)
  if (!tma_out) mdq = mdk = mo;
  static std::atomic<int> slot[kMaxDevices] = {};
  cudaError_t e = ensure_smem(bwd_grads_tc_kernel, GrLay::SMEM_BYTES, slot);
  if (e != cudaSuccess) return e;
  const long long items = (long long)a.NC * a.H;
  const int ctas = (int)(items < device_sm_count() ? items : device_sm_count());
  bwd_grads_tc_kernel<<<ctas, kGrThreads, GrLay::SMEM_BYTES, st>>>(
      mk, mq, mo, static_cast<const __nv_bfloat16*>(a.v), a.g, a.beta, a.UV, a.YX, a.hs, a.dhs,
      static_cast<__nv_bfloat16*>(a.dq), static_cast<__nv_bfloat16*>(a.dk),
      static_cast<__nv_bfloat16*>(a.dv), a.dg, a.dbeta, a.dqk, a.cu, a.coff, a.n_seqs, rows, a.T,
      a.H, a.Hk, (a.T + C - 1) / C, a.hb, a.dhb, mvp, mdx, mdq, mdk, tma_out ? 1 : 0);
  return cudaGetLastError();
}

}  // namespace gdn
