// Per-chunk preparation of the backward on the 5th-generation tensor cores,
// sm_100a: bf16 inputs, dk = dv = 128, dense rows or packed sequences (exact
// semantics).
//
// The backward (chunk_bwd.cu) needs, per chunk of C = 64 tokens and value
// head, with T = (I + A)^{-1}, A = tril_{-1}(beta_i e^{G_i-G_j} K K^T),
// P = tril_0(e^{G_i-G_j} Q K^T), e = e^G, d = e^{G_C - G}:
//
//   W = T diag(beta e) K     U = T diag(beta) V     [C x dk], [C x dv]
//   Z = T^T diag(d) K        Y = T^T P^T dO
//
// in fp32 in its workspace, for its two sequential state passes and its
// per-chunk gradient kernel.  This kernel replaces the warp-level
// preparation (bwd_prep_kernel) at these shapes.  It is the reverse-mode
// counterpart of the recompute_w_u step the reference differentiates through
// (ops.py:276-297, under jax.grad of the chunk path ops.py:299-346).
//
// Tokens past the end of a chunk's sequence (a partial last chunk) take no
// part: their gates are zero, their rows of P and of Z are set to zero, and the
// rest of W, U, Y vanishes with them (beta = 0, identity rows of T).
//
// Persistent, one CTA per SM, one (chunk, head) item at a time:
//   warp 0     TMA loads of K, Q, V, dO (two stages), tcgen05 products, commits
//   warp 1     gate vectors, one item ahead
//   warps 2-9  A and P from the first product, the solve of T (shared with the
//              forward's preparation, chunk_common.cuh), the B operands, and
//              the epilogues that store W, Z, U, Y from TMEM
// Products (tcgen05.mma kind::f16, M = 128, fp32 accumulation in TMEM):
//   D_pre = [K;Q] K^T                       rows 0-63 K K^T, rows 64-127 Q K^T
//   PT    = [T;P] T                         rows 64-127 P T
//   W^T   = K^T (T diag(beta e))^T          M = dk: the transpose sits in TMEM
//   Z^T   = K^T (diag(d) T)                 lane = key dimension, column =
//   U^T   = V^T (T diag(beta))^T            token, so that each epilogue
//   Y^T   = dO^T (P T)                      store of a warp is 128 B wide
// Operands are bf16 (T, P T and the scaled T tiles rounded once), the
// accumulation fp32.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "chunk_common.cuh"
#include "gdn_common.cuh"
#include "gdn_internal.h"
#include "ptx.cuh"

namespace gdn {

namespace {

constexpr int BP_DK = 128, BP_DV = 128;
constexpr int kBpThreads = 320;

// Shared memory from a 1024-byte aligned base.  A stage holds one item's
// inputs: two 64-column key blocks of [K (8 KB) | Q (8 KB)], then V and dO in
// two 64-column blocks of 8 KB each.
struct BpLay {
  static constexpr int STAGE = 65536;
  static constexpr int ST_KQ = 0, ST_V = 32768, ST_DO = 49152;
  static constexpr int SM_AF = 2 * STAGE;               // fp32 A [64][LDF]
  static constexpr int SM_TF = SM_AF + 64 * LDF * 4;    // fp32 T scratch [64][LDF]
  static constexpr int SM_TP = SM_TF + 64 * LDF * 4;    // bf16 [T; P], 128 rows (K-major)
  static constexpr int SM_TD = SM_TP + 16384;           // bf16 diag(d) T  (rows j)
  static constexpr int SM_TB = SM_TD + 8192;            // bf16 T diag(beta)   (rows i)
  static constexpr int SM_TBE = SM_TB + 8192;           // bf16 T diag(beta e) (rows i)
  static constexpr int SM_PTT = SM_TBE + 8192;          // bf16 P T (rows j)
  static constexpr int SM_VEC = SM_PTT + 8192;          // 2 x VecBuf
  static constexpr int SM_BAR = SM_VEC + 2 * (int)sizeof(VecBuf);
  static constexpr int SM_TMEM = SM_BAR + 16 * 8;
  static constexpr int SMEM_BYTES = SM_TMEM + 16 + 1024;
  static_assert(SM_AF % 1024 == 0 && SM_TF % 1024 == 0 && SM_TP % 1024 == 0 &&
                    SM_TD % 1024 == 0 && SM_TB % 1024 == 0 && SM_TBE % 1024 == 0 &&
                    SM_PTT % 1024 == 0,
                "swizzled tiles");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
};

enum {
  B_FULL = 0,     // [2] an item's K, Q, V, dO landed (by stage)
  B_PRE = 2,      // [2] the item's first product in TMEM (by stage)
  B_VFULL = 4,    // [2] gate vectors ready
  B_VEMPTY = 6,   // [2] gate vectors read
  B_TP = 8,       // T, P and the scaled T tiles written
  B_MMA1 = 9,     // P T, W^T, Z^T, U^T in TMEM
  B_PTT = 10,     // the P T tile written (4 warps)
  B_MMA2 = 11,    // Y^T in TMEM: every product of the item complete
};

// TMEM columns (the CTA has the SM to itself): two first-product buffers,
// then one 64-column accumulator per product.
constexpr uint32_t BT_PRE = 0, BT_PT = 128, BT_W = 192, BT_Z = 256, BT_U = 320, BT_Y = 384,
                   BT_COLS = 512;

constexpr uint32_t IDESC_MK = idesc_bf16(128, 64, 1, 0);  // A MN-major, B K-major

__global__ void __launch_bounds__(kBpThreads, 1)
bwd_prep_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmQ,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                   const float* __restrict__ g, const float* __restrict__ beta,
                   float* __restrict__ Wg, float* Zg, float* __restrict__ Ug,
                   float* __restrict__ Yg, const int* __restrict__ cu,
                   const int* __restrict__ coff, int n_seqs, int B, int T, int H, int Hk,
                   int N) {
  using L = BpLay;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  unsigned char* sm = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::SM_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + L::SM_TMEM);
  VecBuf* vecs = reinterpret_cast<VecBuf*>(sm + L::SM_VEC);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool wu = Wg != nullptr;   // W and U wanted (the warp-level forward pass reads them)
  // Items w = blockIdx.x + j gridDim.x: value head h = w % H of global chunk
  // gc = w / H, whose workspace rows are (gc H + h) C ...  Dense: chunk n of
  // row b is gc = b N + n.  Packed (n_seqs > 0): B = 1 row of T tokens, and
  // sequence s owns the chunks coff[s] .. coff[s + 1] - 1 (offsets written by
  // the launch before this one on the stream).
  const long long total = (long long)(n_seqs ? coff[n_seqs] : B * N) * H;
  const int cnt = blockIdx.x < total ? (int)((total - 1 - blockIdx.x) / gridDim.x) + 1 : 0;
  struct Item {
    int gc, h, hq, b, tok, len;   // tok: first token of the chunk in row b; len: its tokens
  };
  const bool small = total < (1LL << 31);
  auto item = [&](int j) {
    const long long w = blockIdx.x + (long long)j * gridDim.x;
    Item it;
    if (small) {   // (32-bit division: the 64-bit one is a long software sequence)
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
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[B_FULL + i], 1);
      mbar_init(&bars[B_PRE + i], 1);
      mbar_init(&bars[B_VFULL + i], 1);
      mbar_init(&bars[B_VEMPTY + i], 1);
    }
    mbar_init(&bars[B_TP], 1);
    mbar_init(&bars[B_MMA1], 1);
    mbar_init(&bars[B_PTT], 4);
    mbar_init(&bars[B_MMA2], 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, BT_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sbase = smem_u32(sm);

  if (warp == 0) {
    // ---- loads and products ----
    if (lane == 0 && cnt > 0) {
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmV);
      prefetch_tmap(&tmO);
      auto load = [&](int j) {
        const Item it = item(j);
        unsigned char* st = sm + (j & 1) * L::STAGE;
        uint64_t* fb = &bars[B_FULL + (j & 1)];
        mbar_arrive_expect_tx(fb, (uint32_t)L::STAGE);
        for (int kb = 0; kb < 2; ++kb) {
          tma_load_4d(st + L::ST_KQ + kb * 16384, &tmK, 64 * kb, it.hq, it.tok, it.b, fb);
          tma_load_4d(st + L::ST_KQ + kb * 16384 + 8192, &tmQ, 64 * kb, it.hq, it.tok, it.b, fb);
          tma_load_4d(st + L::ST_V + kb * 8192, &tmV, 64 * kb, it.h, it.tok, it.b, fb);
          tma_load_4d(st + L::ST_DO + kb * 8192, &tmO, 64 * kb, it.h, it.tok, it.b, fb);
        }
      };
      // D_pre = [K;Q] K^T (K-dim = dk: 8 steps of 16)
      auto first_product = [&](int j) {
        const uint32_t kq = sbase + (uint32_t)(j & 1) * L::STAGE + L::ST_KQ;
#pragma unroll
        for (int k = 0; k < BP_DK / 16; ++k) {
          const uint32_t off = (k >> 2) * 16384 + (k & 3) * 32;
          mma_bf16(tmem + BT_PRE + (uint32_t)(j & 1) * 64, umma_desc(kq + off, 16, 1024, SW128),
                   umma_desc(kq + off, 16, 1024, SW128), IDESC_KK, k > 0);
        }
        mma_commit(&bars[B_PRE + (j & 1)]);
      };
      load(0);
      if (cnt > 1) load(1);
      int issued = cnt < 2 ? cnt : 2;   // items whose loads were issued
      int landed = 0;                   // items whose loads were seen to land
      bool ok = mbar_wait(&bars[B_FULL], 0);
      if (ok) {
        landed = 1;
        tc_fence_after();
        first_product(0);
      }
      for (int j = 0; j < cnt && ok; ++j) {
        const int s = j & 1;
        const uint32_t st = sbase + (uint32_t)s * L::STAGE;
        ok = mbar_wait(&bars[B_TP], (uint32_t)j & 1u);
        if (!ok) break;
        tc_fence_after();
        // P T: [T;P] T (A K-major over the chunk's tokens; B = T, MN-major)
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + BT_PT, umma_desc(sbase + L::SM_TP + k * 32, 16, 1024, SW128),
                   umma_desc(sbase + L::SM_TP + k * 2048, 8192, 1024, SW128), IDESC_KM, k > 0);
        // W^T = K^T (T diag(beta e))^T and Z^T = K^T (diag(d) T): A = K^T,
        // MN-major, M = dk in two 64-wide blocks 16 KB apart
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t a = umma_desc(st + L::ST_KQ + k * 2048, 16384, 1024, SW128);
          if (wu)
            mma_bf16(tmem + BT_W, a, umma_desc(sbase + L::SM_TBE + k * 32, 16, 1024, SW128),
                     IDESC_MK, k > 0);
          mma_bf16(tmem + BT_Z, a, umma_desc(sbase + L::SM_TD + k * 2048, 8192, 1024, SW128),
                   IDESC_MM, k > 0);
        }
        // U^T = V^T (T diag(beta))^T: A = V^T, M = dv in two blocks 8 KB apart
        if (wu) {
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_bf16(tmem + BT_U, umma_desc(st + L::ST_V + k * 2048, 8192, 1024, SW128),
                     umma_desc(sbase + L::SM_TB + k * 32, 16, 1024, SW128), IDESC_MK, k > 0);
        }
        mma_commit(&bars[B_MMA1]);
        // the next item's first product (its buffer's last reader, this
        // item's A/P pass, finished before B_TP)
        if (j + 1 < cnt) {
          ok = mbar_wait(&bars[B_FULL + (s ^ 1)], (uint32_t)((j + 1) >> 1) & 1u);
          if (!ok) break;
          landed = j + 2;
          tc_fence_after();
          first_product(j + 1);
        }
        // Y^T = dO^T (P T), once the P T tile is in shared memory
        ok = mbar_wait(&bars[B_PTT], (uint32_t)j & 1u);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + BT_Y, umma_desc(st + L::ST_DO + k * 2048, 8192, 1024, SW128),
                   umma_desc(sbase + L::SM_PTT + k * 2048, 8192, 1024, SW128), IDESC_MM, k > 0);
        mma_commit(&bars[B_MMA2]);
        // every product of this item has read its stage: load item j + 2 there
        if (j + 2 < cnt) {
          ok = mbar_wait(&bars[B_MMA2], (uint32_t)j & 1u);
          if (!ok) break;
          load(j + 2);
          issued = j + 3;
        }
      }
      // every issued load lands before the CTA can exit (bounded)
      for (int j = landed; j < issued; ++j)
        mbar_wait(&bars[B_FULL + (j & 1)], (uint32_t)(j >> 1) & 1u);
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
      if (j >= 2 && !mbar_wait(&bars[B_VEMPTY + s], (uint32_t)((j - 2) >> 1) & 1u)) break;
      chunk_gate_vectors(vecs[s], g0, g1, b0, b1, true, lane);
      if (lane == 0) mbar_arrive(&bars[B_VFULL + s]);
      if (j + 1 < cnt) fetch(j + 1);
    }
  } else {
    // ---- the math warps ----
    const int pw = warp - 2;          // 0..7
    const int pi = tid - 64;          // 0..255
    const int wq = warp & 3;          // TMEM lane quarter this warp may read
    const int ch = pw >> 2;           // which 32 of 64 accumulator columns
    const int p = wq * 32 + lane;     // TMEM lane
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    float* AF = reinterpret_cast<float*>(sm + L::SM_AF);
    float* TF = reinterpret_cast<float*>(sm + L::SM_TF);
    unsigned char* tpt = sm + L::SM_TP;
    unsigned char* tdt = sm + L::SM_TD;
    // The strictly upper 16x16 blocks of T and diag(d) T are never written below.
    for (int e = pi; e < 64 * 8; e += 256) {
      const int row = e / 8, c8 = e % 8;
      if (c8 >= 2 * (row / 16 + 1)) {
        *reinterpret_cast<uint4*>(tpt + sw128(row, c8)) = make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(tdt + sw128(row, c8)) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    bool ok = true;
    for (int j = 0; j < cnt; ++j) {
      const int s = j & 1;
      const Item it = item(j);
      const size_t row0 = ((size_t)it.gc * H + it.h) * C;
      const VecBuf& vb = vecs[s];
      ok = mbar_wait(&bars[B_VFULL + s], (uint32_t)(j >> 1) & 1u) && ok;
      ok = mbar_wait(&bars[B_PRE + s], (uint32_t)(j >> 1) & 1u) && ok;
      tc_fence_after();
      // A (rows 0-63 of D_pre, strictly lower) and P (rows 64-127, lower with
      // the diagonal): this warp's 32 columns of row p
      const bool isA = p < 64;
      const int i = p & 63;
      {
        float row[32];
        const int jmax = isA ? i - 1 : (i < it.len ? i : -1);   // P: rows in the sequence
        const float rs = isA ? vb.beta[i] : 1.f;
        const float Gi = vb.G[i];
        tmem_ld32(tmem + BT_PRE + (uint32_t)s * 64 + (uint32_t)ch * 32 + lane_off, row);
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          const int q4 = 2 * ch + h2;
          if (vb.direct) {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const int jj = q4 * 16 + e;
              row[16 * h2 + e] = (jj <= jmax) ? rs * gate_exp(Gi - vb.G[jj]) * row[16 * h2 + e]
                                              : 0.f;
            }
          } else {
            const float fq = rs * vb.F[i][q4];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const int jj = q4 * 16 + e;
              row[16 * h2 + e] = (jj <= jmax) ? fq * vb.E[jj] * row[16 * h2 + e] : 0.f;
            }
          }
        }
        if (isA) {
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            *reinterpret_cast<float4*>(AF + i * LDF + 32 * ch + e) = make_float4(
                rtf32(row[e]), rtf32(row[e + 1]), rtf32(row[e + 2]), rtf32(row[e + 3]));
        } else {
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8)
            *reinterpret_cast<uint4*>(tpt + sw128(64 + i, 4 * ch + c8)) = pack_bf16x8(row + 8 * c8);
        }
      }
      // ---- T = (I + A)^{-1}: diagonal blocks, then off-diagonal blocks ----
      if (!named_sync_and(1, 256, ok)) break;
      if (pi < 64) solve_diag(AF, TF, tpt, nullptr, vb.dec, pi);
      named_sync(1, 256);
      solve_offdiag(AF, TF, tpt, nullptr, vb.dec, pw, lane, 1, 256);
      named_sync(1, 256);
      {
        // the B operands from the bf16 T, row r = pi / 4, 16 columns:
        // diag(d) T (rows scaled), T diag(beta), T diag(beta e) (columns scaled)
        const int r = pi >> 2, c8 = 2 * (pi & 3);
        const float d = vb.dec[r];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          float t8[8], a8[8], b8[8];
          unpack_bf16x8(*reinterpret_cast<const uint4*>(tpt + sw128(r, c8 + u)), t8);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int col = 8 * (c8 + u) + e;
            const float bc = vb.beta[col];
            a8[e] = t8[e] * bc;
            b8[e] = t8[e] * bc * vb.eG[col];
            t8[e] *= d;
          }
          *reinterpret_cast<uint4*>(tdt + sw128(r, c8 + u)) = pack_bf16x8(t8);
          *reinterpret_cast<uint4*>(sm + L::SM_TB + sw128(r, c8 + u)) = pack_bf16x8(a8);
          *reinterpret_cast<uint4*>(sm + L::SM_TBE + sw128(r, c8 + u)) = pack_bf16x8(b8);
        }
      }
      fence_proxy_async_smem();
      named_sync(1, 256);
      if (pi == 0) {
        mbar_arrive(&bars[B_TP]);
        mbar_arrive(&bars[B_VEMPTY + s]);
      }
      ok = mbar_wait(&bars[B_MMA1], (uint32_t)j & 1u) && ok;
      tc_fence_after();
      if (wq >= 2) {
        // the P T tile (row j = p - 64), the B operand of Y^T
        float pt[32];
        tmem_ld32(tmem + BT_PT + (uint32_t)ch * 32 + lane_off, pt);
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8)
          *reinterpret_cast<uint4*>(sm + L::SM_PTT + sw128(p - 64, 4 * ch + c8)) =
              pack_bf16x8(pt + 8 * c8);
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[B_PTT]);
      }
      // W, Z (lane p = key dimension) and U (lane p = value column), tokens
      // 32 ch .. 32 ch + 31: one 128-byte row segment per store of the warp
      {
        float x[32];
        if (wu) {
          tmem_ld32(tmem + BT_W + (uint32_t)ch * 32 + lane_off, x);
#pragma unroll
          for (int e = 0; e < 32; ++e) Wg[(row0 + 32 * ch + e) * BP_DK + p] = x[e];
        }
        tmem_ld32(tmem + BT_Z + (uint32_t)ch * 32 + lane_off, x);
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          if (32 * ch + e >= it.len) x[e] = 0.f;
          Zg[(row0 + 32 * ch + e) * BP_DK + p] = x[e];
        }
        if (wu) {
          tmem_ld32(tmem + BT_U + (uint32_t)ch * 32 + lane_off, x);
#pragma unroll
          for (int e = 0; e < 32; ++e) Ug[(row0 + 32 * ch + e) * BP_DV + p] = x[e];
        }
        ok = mbar_wait(&bars[B_MMA2], (uint32_t)j & 1u) && ok;
        tc_fence_after();
        tmem_ld32(tmem + BT_Y + (uint32_t)ch * 32 + lane_off, x);
#pragma unroll
        for (int e = 0; e < 32; ++e) Yg[(row0 + 32 * ch + e) * BP_DV + p] = x[e];
      }
      tc_fence_before();
      if (!ok) break;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, BT_COLS);
  }
}

}  // namespace

GDN_DEVICE_ERROR_ACCESSOR(device_error_bwd_prep)

bool bwd_prep_tc_supported(int dtype, int dk, int dv) {
  return dtype == kBF16 && dk == BP_DK && dv == BP_DV && encode_fn() != nullptr;
}

cudaError_t launch_bwd_prep_tc(const void* q, const void* k, const void* v, const void* dO,
                               const float* g, const float* beta, float* W, float* Z, float* U,
                               float* Y, const int* cu, const int* coff, int n_seqs, int NC,
                               int B, int T, int H, int Hk, cudaStream_t st) {
  // W, U: both or neither
  if ((W == nullptr) != (U == nullptr) || !Z || !Y) return cudaErrorInvalidValue;
  const int rows = n_seqs ? 1 : B;
  if ((long long)rows * H == 0 || T == 0 || NC == 0) return cudaSuccess;
  CUtensorMap mk, mq, mv, mo;
  if (!make_bf16_map_4d(&mk, k, rows, T, Hk, BP_DK) ||
      !make_bf16_map_4d(&mq, q, rows, T, Hk, BP_DK) ||
      !make_bf16_map_4d(&mv, v, rows, T, H, BP_DV) || !make_bf16_map_4d(&mo, dO, rows, T, H, BP_DV))
    return cudaErrorInvalidValue;
  static std::atomic<int> slot[kMaxDevices] = {};
  cudaError_t e = ensure_smem(bwd_prep_tc_kernel, BpLay::SMEM_BYTES, slot);
  if (e != cudaSuccess) return e;
  // NC: the chunks of every row (packed: an upper bound; the kernel reads the
  // exact count from coff[n_seqs])
  const long long items = (long long)NC * H;
  const int ctas = (int)(items < device_sm_count() ? items : device_sm_count());
  bwd_prep_tc_kernel<<<ctas, kBpThreads, BpLay::SMEM_BYTES, st>>>(
      mk, mq, mv, mo, g, beta, W, Z, U, Y, cu, coff, n_seqs, rows, T, H, Hk,
      (T + C - 1) / C);
  return cudaGetLastError();
}

}  // namespace gdn
