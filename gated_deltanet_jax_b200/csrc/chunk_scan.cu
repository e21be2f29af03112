// Chunked gated delta-rule forward in two launches, sm_100a: a preparation
// kernel over every (chunk, head) pair, then a scan kernel over the chunks of
// each (head, 64-column state tile).
//
// Replaces chunk_gated_delta_rule_fwd (ops.py:299-346) for bf16 inputs with
// dk = 128, dv a multiple of 64, dense rows (exact semantics, chunks of 64).
// The reference computes A, inv(I - A), W and U for every chunk with batched
// XLA ops (ops.py:249-297) and then runs a lax.scan over the chunks
// (ops.py:322-341).  Here the state-independent work is moved into its own,
// fully parallel launch, and the sequential scan keeps only two tensor-core
// round trips per chunk.
//
// Per chunk n (C = 64 tokens, in-chunk cumulative gate G, gamma = e^{G_C},
// dec = e^{G_C - G}):
//
//   preparation (chunk_prep_kernel, persistent, two CTAs per SM, one item per
//   (n, b, h)):
//     D_pre = [K;Q] K^T                           (tcgen05, M = 128)
//     A = tril_{-1}(beta_i e^{G_i-G_j} K K^T),  P = tril_0(e^{G_i-G_j} Q K^T)
//     T = (I + A)^{-1}                            (shared solve, chunk_common.cuh)
//     Z = K^T diag(dec) T   [dk x 64]             (tcgen05: K^T times the tile dec*T)
//     PT = P T              [64 x 64]             (tcgen05: [T;P] times T, rows 64-127)
//     -> 24 KB per chunk-head in the workspace: Z then PT, bf16, in the
//        128-byte-swizzled layout the scan's tensor-core reads take as is
//   scan (chunk_scan_kernel, one CTA per (b, h, 64 state columns)):
//     D1 = [K;Q] S_bf16                           rows 0-63: K S, rows 64-127: Q S
//     X  = beta (V - e^G (K S))                   -> bf16 tile
//     D3 = Z X,  S <- gamma S + D3                (the state increment K^T dec T X)
//     D2 = [Z_hi;PT] X                            rows 64-127: P T X = P V'
//     O  = e^G (Q S) + P T X
//
// This is the recurrence of ops.py:170-184 (V' = T X is the chunk's corrected
// value; the reference's literal chunk path differs, see the CUDA-core kernel).
// The scan's critical path per chunk is D1 -> X -> D3 -> S: two MMA round
// trips and two epilogues, each epilogue spread over eight warps.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "chunk_common.cuh"
#include "gdn_common.cuh"
#include "gdn_internal.h"
#include "ptx.cuh"

namespace gdn {

namespace {

constexpr int DK = 128;
constexpr int DVT = 64;
constexpr int kTileBytes = 24576;  // workspace per chunk-head: Z [128][64] | PT [64][64], bf16
// The backward's tiles: the same, then T [64][64] (bf16, rows as the solve left them)
constexpr int kTileBytesBwd = 32768;

// ---------------------------------------------------------------------------
// preparation kernel
// ---------------------------------------------------------------------------

// Persistent: two CTAs per SM, each walking its share of the (chunk, head)
// items.  Warp 0 loads, issues the MMAs and stores each result; warp 1 forms
// the gate vectors one item ahead; warps 2-9 do the math.  The next item's K
// and Q load while this one is solved (K in two alternating slots, Q in one
// that frees as soon as the item's first product read it), its first product
// runs before this item's result is stored, and the store's read of the
// result tile overlaps the next item's A/P pass (which keeps its rows in
// registers until the tile's space is free).
constexpr int kPrepThreads = 320;

// Shared memory from a 1024-byte aligned base.  Each 64-dimension key block is
// [K slot 0 | Q | K slot 1] (8 KB each): item parity 0 reads [K0; Q] as the
// 128-row operand of its first product, parity 1 reads [Q; K1].  The result
// tile (Z then PT, 24 KB) is written over the fp32 solve scratch.
struct PrepLay {
  static constexpr int KB_STRIDE = 24576;                 // one key block: K0 | Q | K1
  static constexpr int SM_KQ = 0;                         // 2 key blocks, 48 KB
  static constexpr int SM_AF = SM_KQ + 2 * KB_STRIDE;     // fp32 A [64][LDF]
  static constexpr int SM_TF = SM_AF + 64 * LDF * 4;      // fp32 T scratch [64][LDF]
  static constexpr int SM_OUT = SM_AF;                    // Z (16 KB) | PT (8 KB)
  static constexpr int SM_TP = SM_TF + 64 * LDF * 4;      // bf16 [T; P], 128 rows
  static constexpr int SM_TD = SM_TP + 16384;             // bf16 dec * T, 64 rows
  static constexpr int SM_VEC = SM_TD + 8192;             // 2 x VecBuf
  static constexpr int SM_BAR = SM_VEC + 2 * (int)sizeof(VecBuf);
  static constexpr int SM_TMEM = SM_BAR + 16 * 8;
  static constexpr int SMEM_BYTES = SM_TMEM + 16 + 1024;  // + alignment slack
  static_assert(SM_AF % 1024 == 0 && SM_TP % 1024 == 0 && SM_TD % 1024 == 0, "tiles");
  static_assert(2 * 64 * LDF * 4 >= kTileBytes, "result tile over the solve scratch");
  static_assert(2 * (SMEM_BYTES + 1024) <= 228 * 1024, "two CTAs per SM");
};

enum {
  P_FULL = 0,    // [2] K and Q of an item landed (by item parity)
  P_PRE = 2,     // [2] first product of an item in TMEM (by item parity)
  P_VFULL = 4,   // [2] gate vectors ready
  P_VEMPTY = 6,  // [2] gate vectors no longer read
  P_TP = 8,      // T, P, dec T tiles written
  P_MMA = 9,     // PT and Z in TMEM
  P_OUT = 10,    // result tile written (8 warps)
  P_OFREE = 11,  // result tile read by its store: the solve scratch is free again
};

// TMEM columns of a preparation CTA (256 allocated: two CTAs fit one SM)
constexpr uint32_t PT_PRE = 0, PT_PT = 128, PT_Z = 192, PT_COLS = 256;

// kT: the backward's tiles, [Z | PT | T] in 32 KB slots (T copied out of the
// [T; P] operand tile by a second bulk copy of the same group).
template <bool kT>
__global__ void __launch_bounds__(kPrepThreads, 2)
chunk_prep_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmQ,
                  const float* __restrict__ g, const float* __restrict__ beta,
                  unsigned char* __restrict__ ws, int T, int H, int Hk, int BH, int N) {
  using L = PrepLay;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  unsigned char* sm = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::SM_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + L::SM_TMEM);
  VecBuf* vecs = reinterpret_cast<VecBuf*>(sm + L::SM_VEC);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Items w = blockIdx.x + j gridDim.x, last chunks first: what the scan reads
  // first was written last, and is the likeliest to still sit in L2.
  const long long total = (long long)BH * N;
  const int cnt = blockIdx.x < total
                      ? (int)((total - 1 - blockIdx.x) / gridDim.x) + 1 : 0;
  // (32-bit division where the item count allows: the 64-bit one is a long
  // software sequence)
  const bool small = total < (1LL << 31);
  auto item = [&](int j, int& n, int& b, int& h, int& hq) {
    const long long w = blockIdx.x + (long long)j * gridDim.x;
    int bh;
    if (small) {
      const unsigned w32 = (unsigned)w, q = w32 / (unsigned)BH;
      bh = (int)(w32 - q * (unsigned)BH);
      n = N - 1 - (int)q;
    } else {
      bh = (int)(w % BH);
      n = N - 1 - (int)(w / BH);
    }
    b = bh / H;
    h = bh - b * H;
    hq = h * Hk / H;
    return bh;
  };

  // The scan grid may launch once every CTA here has started: it then takes
  // SMs only as these CTAs finish (its reads of the workspace wait for this
  // whole grid).
  griddep_launch_dependents();
  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[P_FULL + i], 1);
      mbar_init(&bars[P_PRE + i], 1);
      mbar_init(&bars[P_VFULL + i], 1);
      mbar_init(&bars[P_VEMPTY + i], 1);
    }
    mbar_init(&bars[P_TP], 1);
    mbar_init(&bars[P_MMA], 1);
    mbar_init(&bars[P_OUT], 8);
    mbar_init(&bars[P_OFREE], 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, PT_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sbase = smem_u32(sm);

  if (warp == 0) {
    // ---- loads, MMAs, stores ----
    if (lane == 0 && cnt > 0) {
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmQ);
      auto load_k = [&](int j) {
        int n, b, h, hq;
        item(j, n, b, h, hq);
        const int s = j & 1;
        mbar_arrive_expect_tx(&bars[P_FULL + s], 32768);  // K now, Q later
        for (int kb = 0; kb < 2; ++kb)
          tma_load_4d(sm + L::SM_KQ + kb * L::KB_STRIDE + s * 16384, &tmK, 64 * kb, hq, n * C,
                      b, &bars[P_FULL + s]);
      };
      auto load_q = [&](int j) {
        int n, b, h, hq;
        item(j, n, b, h, hq);
        for (int kb = 0; kb < 2; ++kb)
          tma_load_4d(sm + L::SM_KQ + kb * L::KB_STRIDE + 8192, &tmQ, 64 * kb, hq, n * C, b,
                      &bars[P_FULL + (j & 1)]);
      };
      // D_pre = [K;Q] K^T (parity 0) or [Q;K] K^T (parity 1), K-dim = dk
      auto first_product = [&](int j) {
        const int s = j & 1;
        const uint32_t a0 = sbase + L::SM_KQ + (s ? 8192u : 0u);
        const uint32_t b0 = sbase + L::SM_KQ + (s ? 16384u : 0u);
#pragma unroll
        for (int k = 0; k < DK / 16; ++k) {
          const uint32_t off = (k >> 2) * L::KB_STRIDE + (k & 3) * 32;
          mma_bf16(tmem + PT_PRE + (uint32_t)s * 64, umma_desc(a0 + off, 16, 1024, SW128),
                   umma_desc(b0 + off, 16, 1024, SW128), IDESC_KK, k > 0);
        }
        mma_commit(&bars[P_PRE + s]);
      };
      load_k(0);
      load_q(0);
      bool ok = mbar_wait(&bars[P_FULL], 0);
      if (ok) {
        tc_fence_after();
        first_product(0);
      }
      for (int j = 0; j < cnt && ok; ++j) {
        const int s = j & 1;
        const bool next = j + 1 < cnt;
        int n, b, h, hq;
        const int bh = item(j, n, b, h, hq);
        // the other K slot was last read by item j - 1's Z, complete by now
        // (its result was written, so the math warps saw it complete)
        if (next) load_k(j + 1);
        // Q is free once this item's first product completed
        ok = mbar_wait(&bars[P_PRE + s], (uint32_t)(j >> 1) & 1u);
        if (!ok) break;
        if (next) load_q(j + 1);
        ok = mbar_wait(&bars[P_TP], (uint32_t)j & 1u);
        if (!ok) break;
        tc_fence_after();
        // PT: [T;P] T (A K-major over the chunk's tokens; B = T, MN-major)
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + PT_PT, umma_desc(sbase + L::SM_TP + k * 32, 16, 1024, SW128),
                   umma_desc(sbase + L::SM_TP + k * 2048, 8192, 1024, SW128), IDESC_KM, k > 0);
        // Z: K^T (dec T) (A = K^T, MN-major: M = dk in two 64-wide blocks)
        const uint32_t ks = sbase + L::SM_KQ + (s ? 16384u : 0u);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + PT_Z, umma_desc(ks + k * 2048, L::KB_STRIDE, 1024, SW128),
                   umma_desc(sbase + L::SM_TD + k * 2048, 8192, 1024, SW128), IDESC_MM, k > 0);
        mma_commit(&bars[P_MMA]);
        // the next item's first product, before this one's result is stored
        if (next) {
          ok = mbar_wait(&bars[P_FULL + (s ^ 1)], (uint32_t)((j + 1) >> 1) & 1u);
          if (!ok) break;
          tc_fence_after();
          first_product(j + 1);
        }
        ok = mbar_wait(&bars[P_OUT], (uint32_t)j & 1u);
        if (!ok) break;
        constexpr size_t kStride = kT ? kTileBytesBwd : kTileBytes;
        unsigned char* dst = ws + ((size_t)bh * N + n) * kStride;
        bulk_s2g(dst, sm + L::SM_OUT, kTileBytes);
        // (T, rows 0-63 of [T; P]: the next item's solve rewrites them only
        // after the arrival below)
        if (kT) bulk_s2g(dst + kTileBytes, sm + L::SM_TP, 8192);
        bulk_commit();
        bulk_wait_read<0>();
        mbar_arrive(&bars[P_OFREE]);
      }
      bulk_wait<0>();
    }
  } else if (warp == 1) {
    // ---- gate vectors, one item ahead ----
    float g0 = 0.f, g1 = 0.f, b0 = 0.f, b1 = 0.f;
    auto fetch = [&](int j) {
      int n, b, h, hq;
      item(j, n, b, h, hq);
      const size_t gb = (size_t)b * T * H + h;
      const int t = n * C + 2 * lane;
      g0 = t < T ? ldg_f32(g + gb + (size_t)t * H) : 0.f;
      g1 = t + 1 < T ? ldg_f32(g + gb + (size_t)(t + 1) * H) : 0.f;
      b0 = t < T ? ldg_f32(beta + gb + (size_t)t * H) : 0.f;
      b1 = t + 1 < T ? ldg_f32(beta + gb + (size_t)(t + 1) * H) : 0.f;
    };
    if (cnt > 0) fetch(0);
    for (int j = 0; j < cnt; ++j) {
      const int s = j & 1;
      if (j >= 2 && !mbar_wait(&bars[P_VEMPTY + s], (uint32_t)((j - 2) >> 1) & 1u)) break;
      chunk_gate_vectors(vecs[s], g0, g1, b0, b1, true, lane);
      if (lane == 0) mbar_arrive(&bars[P_VFULL + s]);
      if (j + 1 < cnt) fetch(j + 1);
    }
  } else {
    // ---- the math warps: A/P, the solve, the result epilogue ----
    const int pw = warp - 2;          // 0..7
    const int pi = tid - 64;          // 0..255
    const int wq = warp & 3;          // TMEM lane quarter this warp may read
    const int ch = pw >> 2;           // which 32 of the 64 D_pre columns
    const int p = wq * 32 + lane;     // TMEM lane = accumulator row
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    float* AF = reinterpret_cast<float*>(sm + L::SM_AF);
    float* TF = reinterpret_cast<float*>(sm + L::SM_TF);
    unsigned char* tpt = sm + L::SM_TP;
    unsigned char* tdt = sm + L::SM_TD;
    // The strictly upper 16x16 blocks of T (and dec T) are never written below.
    for (int e = pi; e < 64 * 8; e += 256) {
      const int row = e / 8, c8 = e % 8;
      if (c8 >= 2 * (row / 16 + 1)) {
        *reinterpret_cast<uint4*>(tpt + sw128(row, c8)) = make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(tdt + sw128(row, c8)) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    // (a timed-out wait is recorded in the device error word; the math warps
    // agree on it at the first named barrier of the item and leave together,
    // so none of them waits at a barrier the others no longer reach)
    bool ok = true;
    for (int j = 0; j < cnt; ++j) {
      const int s = j & 1;
      const VecBuf& vb = vecs[s];
      ok = mbar_wait(&bars[P_VFULL + s], (uint32_t)(j >> 1) & 1u) && ok;
      ok = mbar_wait(&bars[P_PRE + s], (uint32_t)(j >> 1) & 1u) && ok;
      tc_fence_after();
      // A (strictly lower) and P (lower with the diagonal) from D_pre: this
      // warp's 32 columns of row p, which holds K K^T (A) or Q K^T (P)
      // depending on the item's parity.  Steep gates (direct) form each
      // e^{G_i - G_j} from its own exponent.  The row waits in registers
      // until the previous result tile (over A's scratch) has been read out.
      const bool isA = (p < 64) == (s == 0);
      const int i = p & 63;
      float row[32];
      {
        const int jmax = isA ? i - 1 : i;
        const float rs = isA ? vb.beta[i] : 1.f;
        const float Gi = vb.G[i];
        tmem_ld32(tmem + PT_PRE + (uint32_t)s * 64 + (uint32_t)ch * 32 + lane_off, row);
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
      }
      if (j > 0) ok = mbar_wait(&bars[P_OFREE], (uint32_t)(j - 1) & 1u) && ok;
      if (isA) {
#pragma unroll
        for (int e = 0; e < 32; e += 4)
          *reinterpret_cast<float4*>(AF + i * LDF + 32 * ch + e) =
              make_float4(rtf32(row[e]), rtf32(row[e + 1]), rtf32(row[e + 2]), rtf32(row[e + 3]));
      } else {
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8)
          *reinterpret_cast<uint4*>(tpt + sw128(64 + i, 4 * ch + c8)) = pack_bf16x8(row + 8 * c8);
      }
      // ---- T = (I + A)^{-1}: diagonal blocks, then off-diagonal blocks ----
      if (!named_sync_and(1, 256, ok)) break;
      if (pi < 64) solve_diag(AF, TF, tpt, nullptr, vb.dec, pi);
      named_sync(1, 256);
      solve_offdiag(AF, TF, tpt, nullptr, vb.dec, pw, lane, 1, 256);
      named_sync(1, 256);
      {
        // dec T (the B operand of Z), from the bf16 T: row pi / 4, 16 columns
        const int r = pi >> 2, c8 = 2 * (pi & 3);
        const float d = vb.dec[r];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          float t8[8];
          unpack_bf16x8(*reinterpret_cast<const uint4*>(tpt + sw128(r, c8 + u)), t8);
#pragma unroll
          for (int e = 0; e < 8; ++e) t8[e] *= d;
          *reinterpret_cast<uint4*>(tdt + sw128(r, c8 + u)) = pack_bf16x8(t8);
        }
      }
      fence_proxy_async_smem();
      named_sync(1, 256);
      if (pi == 0) {
        mbar_arrive(&bars[P_TP]);
        mbar_arrive(&bars[P_VEMPTY + s]);
      }
      // ---- result: Z (rows 0-127) and PT (rows 64-127 of the [T;P] T
      //      product), bf16, over the solve scratch ----
      ok = mbar_wait(&bars[P_MMA], (uint32_t)j & 1u) && ok;
      tc_fence_after();
      {
        float z[32];
        tmem_ld32(tmem + PT_Z + (uint32_t)ch * 32 + lane_off, z);
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8)
          *reinterpret_cast<uint4*>(sm + L::SM_OUT + sw128(p, 4 * ch + c8)) =
              pack_bf16x8(z + 8 * c8);
        if (wq >= 2) {
          float pt[32];
          tmem_ld32(tmem + PT_PT + (uint32_t)ch * 32 + lane_off, pt);
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8)
            *reinterpret_cast<uint4*>(sm + L::SM_OUT + 16384 + sw128(p - 64, 4 * ch + c8)) =
                pack_bf16x8(pt + 8 * c8);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[P_OUT]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, PT_COLS);
  }
}

// ---------------------------------------------------------------------------
// scan kernel
// ---------------------------------------------------------------------------

constexpr int kScanThreads = 384;  // warps 0-3 roles, 4-11 epilogues
constexpr int NS = 3;              // K/Q/V stages
constexpr int NR = 3;              // ring of preparation tiles
constexpr int NV = 3;              // ring of gate vectors

// barrier indices
enum {
  S_FULL = 0,                 // [NS] K, Q, V of a chunk loaded
  S_EMPTY = S_FULL + NS,      // [NS] the MMAs are done with a stage (V: epilogue 1 read it before X)
  S_RFULL = S_EMPTY + NS,     // [NR] preparation tile loaded
  S_REMPTY = S_RFULL + NR,    // [NR] preparation tile read by the MMAs
  S_VFULL = S_REMPTY + NR,    // [NV] gate vectors ready
  S_VEMPTY = S_VFULL + NV,    // [NV] gate vectors read by every epilogue warp
  S_D1 = S_VEMPTY + NV,       // D1 in TMEM
  S_X,                        // X tile written (4 warps)
  S_D3,                       // D3 in TMEM
  S_D2,                       // D2 in TMEM
  S_D2FREE,                   // D2 read (4 warps)
  S_S,                        // state tile written (8 warps)
  S_D1FREE,                   // [2] a D1 buffer's Q S rows read (4 warps)
  S_DONE = S_D1FREE + 2,
  S_NBAR,
};

struct ScanVec {
  float beta[C], eG[C];
  float eGC;
  float pad[3];
};

struct ScanLay {
  static constexpr int SM_KQ = 0;                        // NS x [2 key blocks][K | Q] (32 KB)
  static constexpr int SM_V = SM_KQ + NS * 32768;        // NS x [64 tokens][128 B]
  static constexpr int SM_R = SM_V + NS * 8192;          // NR x (Z | PT), 24 KB
  static constexpr int SM_S = SM_R + NR * kTileBytes;    // bf16 state tile [128][128 B]
  static constexpr int SM_X = SM_S + 16384;              // bf16 X [64 tokens][128 B]
  static constexpr int SM_VEC = SM_X + 8192;             // NV x ScanVec
  static constexpr int SM_BAR = SM_VEC + NV * (int)sizeof(ScanVec);
  static constexpr int SM_TMEM = SM_BAR + S_NBAR * 8;
  static constexpr int SMEM_BYTES = SM_TMEM + 16 + 1024;
  static_assert(SM_R % 1024 == 0 && SM_S % 1024 == 0 && SM_X % 1024 == 0, "swizzled tiles");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
};

// TMEM columns of a scan CTA
constexpr uint32_t ST_D1 = 0;    // 2 x 64
constexpr uint32_t ST_D3 = 128;
constexpr uint32_t ST_D2 = 192;
constexpr uint32_t ST_COLS = 256;

// One warp's 32 x 32 fp32 block (lane = row) as bf16 through its staging (32
// rows of 64 bytes, unswizzled) to a tensor store at (x, y) with a 32 x 32 bf16
// map; the staging's previous store has read it first.  Lane l writes its four
// 16-byte pieces in an order rotated by l / 2, so that the eight lanes of each
// store phase hit distinct banks.
__device__ __forceinline__ void stage_store_bf16(unsigned char* stg, const float (&vals)[32],
                                                 const CUtensorMap* map, int x, int y, int lane) {
  if (lane == 0) bulk_wait_read<0>();
  __syncwarp();
  uint4 p[4];
#pragma unroll
  for (int c8 = 0; c8 < 4; ++c8) p[c8] = pack_bf16x8(vals + 8 * c8);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int j = (c + (lane >> 1)) & 3;
    const uint4 w = j == 0 ? p[0] : j == 1 ? p[1] : j == 2 ? p[2] : p[3];
    *reinterpret_cast<uint4*>(stg + lane * 64 + j * 16) = w;
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(map, x, y, stg);
    bulk_commit();
  }
}

// kBwd: the forward pass of the backward (chunk_bwd.cu) instead of the forward
// itself.  Its tiles are the preparation's 32 KB [Z | PT | T] slots
// (chunk_prep_kernel<true>), of which Z and T are loaded, T where the forward
// has PT: D2 = [Z rows 64-127; T] X gives V' = T X in rows 64-127, which the
// epilogue warps on those TMEM lanes store; Q is not loaded and no output is
// formed.  Every chunk's entering state goes
// to hs [(b N + n) H + h][dk][dv] and V' to vp [((b N + n) H + h) C + i][dv]
// (fp32), the layouts of the backward's workspace, through the TMA maps tmHS
// and tmVP: each epilogue warp stages its 32 x 32 block in the Q slots (not
// loaded here) and stores it with one tensor store, instead of 32 separate
// row segments per store instruction.  With hsb, the entering states go out
// instead as the bf16 state tile the chain already holds in shared memory
// (16 KB per chunk and CTA, [dk rows][64 columns], 128-byte swizzled) at
// hsb + ((b N + n) H + h) 32 KB + 16 KB x (column tile): one bulk copy per
// chunk, the layout the tcgen05 gradients kernel loads; and V' goes to vp as
// bf16 rows ([((b N + n) H + h) C + i][dv], tmVP a 32 x 32 bf16 map), the
// operand the gradients take, rounded once.
template <bool kBwd>
__global__ void __launch_bounds__(kScanThreads, 1)
chunk_scan_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmQ,
                  const __grid_constant__ CUtensorMap tmV, const float* __restrict__ g,
                  const float* __restrict__ beta, const unsigned char* __restrict__ ws,
                  const float* h0, __nv_bfloat16* __restrict__ o, float* hT, int T, int H,
                  int Hk, int dv, int ds, const __grid_constant__ CUtensorMap tmHS,
                  const __grid_constant__ CUtensorMap tmVP, unsigned char* __restrict__ hsb) {
  // (h0 and hT may be the same array: each CTA reads its tile of h0 before it
  // writes the same tile of hT)
  // The state has ds columns: dv of them follow v (and give o); with ds = dv +
  // dk the last dk are the transition, the same recurrence started from the
  // identity with v = 0 (no V loads, no output, h0 unused there).  o may be
  // NULL (no output stored).
  using L = ScanLay;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  unsigned char* sm = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::SM_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + L::SM_TMEM);
  ScanVec* vecs = reinterpret_cast<ScanVec*>(sm + L::SM_VEC);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh - b * H;
  const int hq = h * Hk / H;
  const int c0 = blockIdx.x * DVT;
  const bool trans = c0 >= dv;  // a transition tile
  const int N = (T + C - 1) / C;

  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&bars[S_FULL + i], 1);
      mbar_init(&bars[S_EMPTY + i], 1);
    }
    for (int i = 0; i < NR; ++i) {
      mbar_init(&bars[S_RFULL + i], 1);
      mbar_init(&bars[S_REMPTY + i], 1);
    }
    for (int i = 0; i < NV; ++i) {
      mbar_init(&bars[S_VFULL + i], 1);
      mbar_init(&bars[S_VEMPTY + i], 8);
    }
    mbar_init(&bars[S_D1], 1);
    mbar_init(&bars[S_X], 4);
    mbar_init(&bars[S_D3], 1);
    mbar_init(&bars[S_D2], 1);
    mbar_init(&bars[S_D2FREE], 4);
    mbar_init(&bars[S_S], 8);
    mbar_init(&bars[S_D1FREE + 0], 4);
    mbar_init(&bars[S_D1FREE + 1], 4);
    mbar_init(&bars[S_DONE], 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, ST_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sbase = smem_u32(sm);
  // Launched with programmatic stream serialization, the set-up above may
  // overlap the previous kernel on the stream; everything below reads memory
  // that kernel may write (the workspace after the preparation; h0, q, k, v, g,
  // beta after any other), so every thread waits for it to complete here.
  griddep_wait();

  if (warp == 0) {
    // ---- K, Q, V of each chunk (TMA) ----
    if (elect_one()) {
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmV);
      int issued = 0;
      for (int n = 0; n < N; ++n) {
        const int s = n % NS;
        if (n >= NS && !mbar_wait(&bars[S_EMPTY + s], (uint32_t)((n / NS) - 1) & 1u)) break;
        unsigned char* kq = sm + L::SM_KQ + s * 32768;
        uint64_t* fb = &bars[S_FULL + s];
        mbar_arrive_expect_tx(fb, (kBwd ? 16384 : 32768) + (trans ? 0 : 8192));
        for (int kb = 0; kb < 2; ++kb) {
          tma_load_4d(kq + kb * 16384, &tmK, 64 * kb, hq, n * C, b, fb);
          if (!kBwd) tma_load_4d(kq + kb * 16384 + 8192, &tmQ, 64 * kb, hq, n * C, b, fb);
        }
        if (!trans) tma_load_4d(sm + L::SM_V + s * 8192, &tmV, c0, h, n * C, b, fb);
        issued = n + 1;
      }
      // every issued load lands before the CTA can exit (bounded)
      for (int n = issued > NS ? issued - NS : 0; n < issued; ++n)
        mbar_wait(&bars[S_FULL + n % NS], (uint32_t)(n / NS) & 1u);
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (elect_one()) {
      bool ok = true;
      for (int n = 0; n < N && ok; ++n) {
        const int s = n % NS, r = n % NR, buf = n & 1;
        const uint32_t kq = sbase + L::SM_KQ + s * 32768;
        const uint32_t rt = sbase + L::SM_R + r * kTileBytes;
        ok = mbar_wait(&bars[S_FULL + s], (uint32_t)(n / NS) & 1u) &&
             mbar_wait(&bars[S_S], (uint32_t)n & 1u) &&
             (n < 2 || mbar_wait(&bars[S_D1FREE + buf], (uint32_t)((n - 2) >> 1) & 1u));
        if (!ok) break;
        tc_fence_after();
        // D1 = [K;Q] S   (K-dim = dk: 8 steps of 16)
#pragma unroll
        for (int k = 0; k < DK / 16; ++k) {
          const uint64_t a = umma_desc(kq + (k >> 2) * 16384 + (k & 3) * 32, 16, 1024, SW128);
          const uint64_t bd = umma_desc(sbase + L::SM_S + k * 2048, 16384, 1024, SW128);
          mma_bf16(tmem + ST_D1 + (uint32_t)buf * 64, a, bd, IDESC_KM, k > 0);
        }
        mma_commit(&bars[S_D1]);
        if (kBwd && hsb) {
          // the bf16 state entering chunk n, as the tile D1 just read
          bulk_s2g(hsb + (((size_t)b * N + n) * H + h) * kHandoffHSlot + blockIdx.x * 16384,
                   sm + L::SM_S, 16384);
          bulk_commit();
        }
        ok = mbar_wait(&bars[S_X], (uint32_t)n & 1u) &&
             mbar_wait(&bars[S_RFULL + r], (uint32_t)(n / NR) & 1u) &&
             (n < 1 || mbar_wait(&bars[S_D2FREE], (uint32_t)(n - 1) & 1u));
        if (!ok) break;
        // the state tile is rewritten once D3 completes: its copy has read it
        if (kBwd && hsb) bulk_wait_read<0>();
        tc_fence_after();
        // D3 = Z X, the state increment (K-dim = tokens: 4 steps)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t a = umma_desc(rt + k * 32, 16, 1024, SW128);
          const uint64_t bd = umma_desc(sbase + L::SM_X + k * 2048, 8192, 1024, SW128);
          mma_bf16(tmem + ST_D3, a, bd, IDESC_KM, k > 0);
        }
        mma_commit(&bars[S_D3]);
        // D2 = [Z rows 64-127; PT] X: rows 64-127 are P T X (kBwd: [Z rows
        // 64-127; T] X, rows 64-127 are V' = T X)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t a = umma_desc(rt + 8192 + k * 32, 16, 1024, SW128);
          const uint64_t bd = umma_desc(sbase + L::SM_X + k * 2048, 8192, 1024, SW128);
          mma_bf16(tmem + ST_D2, a, bd, IDESC_KM, k > 0);
        }
        mma_commit(&bars[S_D2]);
        mma_commit(&bars[S_EMPTY + s]);
        mma_commit(&bars[S_REMPTY + r]);
      }
      mma_commit(&bars[S_DONE]);
      mbar_wait(&bars[S_DONE], 0);
      if (kBwd && hsb) bulk_wait<0>();
    }
  } else if (warp == 2) {
    // ---- gate warp: beta, e^G and e^{G_C} of each chunk, NV - 1 chunks ahead ----
    const size_t gb = (size_t)b * T * H + h;
    for (int n = 0; n < N; ++n) {
      const int v = n % NV;
      const int t = n * C + 2 * lane;
      const float g0 = t < T ? ldg_f32(g + gb + (size_t)t * H) : 0.f;
      const float g1 = t + 1 < T ? ldg_f32(g + gb + (size_t)(t + 1) * H) : 0.f;
      const float b0 = t < T ? ldg_f32(beta + gb + (size_t)t * H) : 0.f;
      const float b1 = t + 1 < T ? ldg_f32(beta + gb + (size_t)(t + 1) * H) : 0.f;
      if (n >= NV && !mbar_wait(&bars[S_VEMPTY + v], (uint32_t)((n / NV) - 1) & 1u)) break;
      ScanVec& vb = vecs[v];
      const float pair = g0 + g1;
      float incl = pair;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += y;
      }
      vb.beta[2 * lane] = b0;
      vb.beta[2 * lane + 1] = b1;
      vb.eG[2 * lane] = gate_exp(incl - pair + g0);
      vb.eG[2 * lane + 1] = gate_exp(incl);
      if (lane == 31) vb.eGC = gate_exp(incl);
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[S_VFULL + v]);
    }
  } else if (warp == 3) {
    // ---- preparation tiles (bulk copies from the workspace) ----
    if (elect_one()) {
      constexpr size_t kStride = kBwd ? kTileBytesBwd : kTileBytes;
      const unsigned char* src = ws + (size_t)bh * N * kStride;
      int issued = 0;
      for (int n = 0; n < N; ++n) {
        const int r = n % NR;
        if (n >= NR && !mbar_wait(&bars[S_REMPTY + r], (uint32_t)((n / NR) - 1) & 1u)) break;
        mbar_arrive_expect_tx(&bars[S_RFULL + r], kTileBytes);
        if (kBwd) {
          // Z, then T in place of PT
          bulk_g2s(sm + L::SM_R + r * kTileBytes, src + (size_t)n * kStride, 16384,
                   &bars[S_RFULL + r]);
          bulk_g2s(sm + L::SM_R + r * kTileBytes + 16384, src + (size_t)n * kStride + kTileBytes,
                   8192, &bars[S_RFULL + r]);
        } else {
          bulk_g2s(sm + L::SM_R + r * kTileBytes, src + (size_t)n * kStride, kTileBytes,
                   &bars[S_RFULL + r]);
        }
        issued = n + 1;
      }
      for (int n = issued > NR ? issued - NR : 0; n < issued; ++n)
        mbar_wait(&bars[S_RFULL + n % NR], (uint32_t)(n / NR) & 1u);
    }
  } else {
    // ---- epilogue warps: quarter wq of the TMEM lanes, 32 of the 64 columns ----
    const int wq = warp & 3;
    const int cb = 32 * ((warp - 4) >> 2);  // column offset within the tile
    const int r = wq * 32 + lane;           // TMEM lane: state row, or token row
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    unsigned char* Stile = sm + L::SM_S;
    // kBwd staging (4 KB per warp) in the six 8 KB Q slots, which are not loaded:
    // slot p = stage p / 2, key block p % 2.  Epilogue warp e stages its state
    // block in slot e / 2; the four warps on lanes 64-127 their V' block in slots 4-5.
    const int ew = warp - 4;
    auto qslot = [&](int p, int half) {
      return sm + L::SM_KQ + (p >> 1) * 32768 + (p & 1) * 16384 + 8192 + half * 4096;
    };
    unsigned char* stg_s = qslot(ew >> 1, ew & 1);
    const int xw = (wq & 1) + 2 * (cb >> 5);
    unsigned char* stg_v = qslot(4 + (xw >> 1), xw & 1);
    // this warp's 32 x 32 fp32 block (lane = row) through its staging to a
    // tensor store at (x, y); the staging's previous store has read it first
    auto stage_store = [&](unsigned char* stg, const float (&vals)[32], const CUtensorMap* map,
                           int x, int y) {
      if (lane == 0) bulk_wait_read<0>();
      __syncwarp();
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8)
        *reinterpret_cast<float4*>(stg + sw128(lane, c8)) =
            make_float4(vals[4 * c8], vals[4 * c8 + 1], vals[4 * c8 + 2], vals[4 * c8 + 3]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(map, x, y, stg);
        bulk_commit();
      }
    };
    float S[32];
    {
      const float* src = h0 && !trans ? h0 + ((size_t)bh * DK + r) * ds + c0 + cb : nullptr;
#pragma unroll
      for (int c = 0; c < 32; c += 4) {
        const float4 x = src ? *reinterpret_cast<const float4*>(src + c)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
        S[c] = x.x; S[c + 1] = x.y; S[c + 2] = x.z; S[c + 3] = x.w;
      }
      if (trans) {
#pragma unroll
        for (int c = 0; c < 32; ++c) S[c] = (c0 - dv + cb + c == r) ? 1.f : 0.f;
      }
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8)
        *reinterpret_cast<uint4*>(Stile + sw128(r, cb / 8 + c8)) = pack_bf16x8(S + 8 * c8);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[S_S]);
    }
    bool ok = true;
    for (int n = 0; n < N && ok; ++n) {
      const int s = n % NS, v = n % NV, buf = n & 1;
      const ScanVec& vb = vecs[v];
      const uint32_t d1 = tmem + ST_D1 + (uint32_t)buf * 64 + (uint32_t)cb + lane_off;
      // workspace slot of (chunk n, head) in the backward's layout
      const size_t slot = ((size_t)b * N + n) * H + h;
      if (kBwd && !hsb && n == 0) {
        // the state entering chunk 0 (later ones are stored as they are formed)
        stage_store(stg_s, S, &tmHS, c0 + cb, (int)(slot * DK) + wq * 32);
      }
      ok = mbar_wait(&bars[S_VFULL + v], (uint32_t)(n / NV) & 1u);
      if (!ok) break;
      if (wq < 2) {
        // ---- epilogue 1: X = beta (V - e^G K S), token row r ----
        // The row of V (landed with the chunk's K and Q, usually chunks ago)
        // is read into registers before the wait for D1, so that its
        // shared-memory latency overlaps the MMA instead of following it.
        ok = mbar_wait(&bars[S_FULL + s], (uint32_t)(n / NS) & 1u);
        if (!ok) break;
        const unsigned char* Vt = sm + L::SM_V + s * 8192;
        uint4 vrow[4];
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8)
          vrow[c8] = trans ? make_uint4(0u, 0u, 0u, 0u)
                           : *reinterpret_cast<const uint4*>(Vt + sw128(r, cb / 8 + c8));
        const float bi = vb.beta[r], egi = vb.eG[r];
        ok = mbar_wait(&bars[S_D1], (uint32_t)n & 1u);
        if (!ok) break;
        tc_fence_after();
        float ks[32];
        tmem_ld32(d1, ks);
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          float vv[8], x[8];
          unpack_bf16x8(vrow[c8], vv);
#pragma unroll
          for (int e = 0; e < 8; ++e) x[e] = bi * (vv[e] - egi * ks[8 * c8 + e]);
          *reinterpret_cast<uint4*>(sm + L::SM_X + sw128(r, cb / 8 + c8)) = pack_bf16x8(x);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[S_X]);
      }
      // ---- epilogue 3: S <- e^{G_C} S + Z X, state row r ----
      ok = mbar_wait(&bars[S_D3], (uint32_t)n & 1u);
      if (!ok) break;
      tc_fence_after();
      {
        float ds[32];
        tmem_ld32(tmem + ST_D3 + (uint32_t)cb + lane_off, ds);
        const float egc = vb.eGC;
#pragma unroll
        for (int e = 0; e < 32; ++e) S[e] = fmaf(egc, S[e], ds[e]);
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8)
          *reinterpret_cast<uint4*>(Stile + sw128(r, cb / 8 + c8)) = pack_bf16x8(S + 8 * c8);
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[S_S]);
        if (kBwd && !hsb && n + 1 < N) {
          // the state entering chunk n + 1, after the arrival
          stage_store(stg_s, S, &tmHS, c0 + cb, (int)((slot + H) * DK) + wq * 32);
        }
      }
      if constexpr (kBwd) {
        if (wq >= 2) {
          // ---- V' = T X (rows 64-127 of D2), token row r - 64, into vp ----
          ok = mbar_wait(&bars[S_D2], (uint32_t)n & 1u);
          if (!ok) break;
          tc_fence_after();
          float x[32];
          tmem_ld32(tmem + ST_D2 + (uint32_t)cb + lane_off, x);
          tc_fence_before();
          __syncwarp();
          // (no output: the D1 buffer's Q rows are not read)
          if (lane == 0) {
            mbar_arrive(&bars[S_D2FREE]);
            mbar_arrive(&bars[S_D1FREE + buf]);
          }
          // stored after the arrival, which gates the next chunk's products
          // (rows past T hold V' = 0: their X is zero)
          const int row = (int)(slot * C) + (wq - 2) * 32;
          if (hsb)
            stage_store_bf16(stg_v, x, &tmVP, c0 + cb, row, lane);
          else
            stage_store(stg_v, x, &tmVP, c0 + cb, row);
        }
      } else if (wq >= 2) {
        // ---- output: O = e^G (Q S) + P T X, token row r - 64 ----
        ok = mbar_wait(&bars[S_D2], (uint32_t)n & 1u);
        if (!ok) break;
        tc_fence_after();
        const int i = r - 64, t = n * C + i;
        float qs[16], pv[16];
        const float egi = vb.eG[i];
        __nv_bfloat16* orow =
            o && !trans ? o + (((size_t)b * T + t) * H + h) * dv + c0 + cb : nullptr;
#pragma unroll
        for (int q2 = 0; q2 < 2; ++q2) {
          tmem_ld16x2(d1 + 16 * q2, tmem + ST_D2 + (uint32_t)cb + lane_off + 16 * q2, qs, pv);
          float out[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) out[e] = fmaf(egi, qs[e], pv[e]);
          if (t < T && orow) {
            *reinterpret_cast<uint4*>(orow + 16 * q2) = pack_bf16x8(out);
            *reinterpret_cast<uint4*>(orow + 16 * q2 + 8) = pack_bf16x8(out + 8);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&bars[S_D2FREE]);
          mbar_arrive(&bars[S_D1FREE + buf]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[S_VEMPTY + v]);
    }
    if (ok && hT) {
      float* dst = hT + ((size_t)bh * DK + r) * ds + c0 + cb;
#pragma unroll
      for (int c = 0; c < 32; c += 4)
        *reinterpret_cast<float4*>(dst + c) = make_float4(S[c], S[c + 1], S[c + 2], S[c + 3]);
    }
    if (kBwd && lane == 0) bulk_wait<0>();   // every tensor store done before exit
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, ST_COLS);
  }
}

// ---------------------------------------------------------------------------
// reverse scan: the backward's reverse state pass
// ---------------------------------------------------------------------------

// The backward's reverse pass (chunk_bwd.cu) walks the chunks from the last
// to the first with the gradient R of the state leaving the chunk (starting
// from dhT), per (b, h, 64 state columns), with Z = T^T diag(d) K and PT = P T
// from the preparation's [Z | PT | T] slots (chunk_prep_kernel<true>):
//   D1 = PT^T dO + Z R            (tcgen05: A = PT^T and Z read MN-major from
//                                  the tiles as stored; the dO product, which
//                                  does not depend on R, is issued first)
//   dX = D1                       -> yx (fp32)
//   X  = -beta e dX               -> bf16 tile
//   D3 = Q^T (e dO) + K^T X       (tcgen05, K-dim 128: the dO half is issued
//                                  before X is known)
//   R <- e^{G_C} R + D3           -> every chunk's leaving gradient to dhs
// the reverse of the warp-level bwd_states_kernel's second direction, on the
// same two-round-trip chain as the forward scan.  dX (rows of yx) and
// the leaving gradients (rows of dhs) go out by TMA tensor stores (tmYX,
// tmDHS), each epilogue warp staging its 32 x 32 block; with dhsb the
// gradients go out instead as the bf16 tile the chain holds (one bulk copy
// per chunk, the layout of the forward scan's hsb).  Loads per chunk: K, Q (TMA),
// dO (TMA, this CTA's 64 columns) and the first 24 KB ([Z | PT]) of the
// preparation's slot.  The epilogue warps on TMEM lanes 64-127 form e dO for the products.
// With dhsb (the hand-off to the tcgen05 gradients) the CTA also loads its 64
// columns of v and, from each token row's fp32 dX, writes dV = beta dX (dvo),
// the row's partial sum of dX o v over its 32 columns (fp32, at dhsb + 36 KB x
// slot + 32 KB, [64 tokens][4 column blocks]), and dX as bf16 rows through
// tmYX (a 32 x 32 bf16 map) instead of fp32.
constexpr int kRevTile = 24576;   // Z [128 keys][64 tokens] | PT [64][64], bf16
constexpr int kRevNR = 2;         // ring of [Z | PT] tiles
constexpr int kRevNS = 2;         // K/Q/dO stages (the rest of shared memory stages the stores)

struct RevLay {
  static constexpr int SM_KQ = 0;                          // kRevNS x [2 key blocks][K | Q]
  static constexpr int SM_DO = SM_KQ + kRevNS * 32768;     // kRevNS x dO [64 tokens][128 B]
  static constexpr int SM_Z = SM_DO + kRevNS * 8192;       // kRevNR x [Z | PT]
  static constexpr int SM_S = SM_Z + kRevNR * kRevTile;    // bf16 gradient tile [128][128 B]
  static constexpr int SM_X = SM_S + 16384;                // bf16 -beta e dX [64][128 B]
  static constexpr int SM_E = SM_X + 8192;                 // bf16 e dO [64][128 B]
  static constexpr int SM_STG = SM_E + 8192;               // 12 x 4 KB store staging
  static constexpr int SM_V = SM_STG;   // with dhsb: kRevNS x v [64 tokens][128 B] (slots 0-3)
  static constexpr int SM_VEC = SM_STG + 12 * 4096;        // NV x ScanVec
  static constexpr int SM_BAR = SM_VEC + NV * (int)sizeof(ScanVec);
  static constexpr int SM_TMEM = SM_BAR + 32 * 8;
  static constexpr int SMEM_BYTES = SM_TMEM + 16 + 1024;
  static_assert(SM_Z % 1024 == 0 && SM_S % 1024 == 0 && SM_X % 1024 == 0 && SM_E % 1024 == 0 &&
                    SM_STG % 1024 == 0,
                "swizzled tiles");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
};

enum {
  R_FULL = 0,                 // [kRevNS] K, Q, dO of a chunk loaded
  R_EMPTY = R_FULL + kRevNS,  // [kRevNS] its products done, its dO read
  R_ZFULL = R_EMPTY + kRevNS,     // [kRevNR] Z | PT tile loaded
  R_ZEMPTY = R_ZFULL + kRevNR,    // [kRevNR] Z | PT tile read
  R_VFULL = R_ZEMPTY + kRevNR,    // [NV] gate vectors ready
  R_VEMPTY = R_VFULL + NV,    // [NV] gate vectors read (8 warps)
  R_D1 = R_VEMPTY + NV,       // D1 in TMEM
  R_X,                        // X tile written (4 warps)
  R_E,                        // e dO tile written (4 warps)
  R_D3,                       // D3 in TMEM
  R_S,                        // gradient tile written (8 warps)
  R_D1FREE,                   // [2] a D1 buffer read (4 warps)
  R_DONE = R_D1FREE + 2,
  R_NBAR,
};
static_assert(R_NBAR <= 32, "barrier space");

__global__ void __launch_bounds__(kScanThreads, 1)
chunk_scan_rev_kernel(const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmQ,
                      const __grid_constant__ CUtensorMap tmO, const float* __restrict__ g,
                      const float* __restrict__ beta, const unsigned char* __restrict__ tiles,
                      const float* __restrict__ dhT, float* __restrict__ dh0,
                      const __grid_constant__ CUtensorMap tmYX,
                      const __grid_constant__ CUtensorMap tmDHS, unsigned char* __restrict__ dhsb,
                      const __grid_constant__ CUtensorMap tmV, __nv_bfloat16* __restrict__ dvo,
                      int T, int H, int Hk, int dv) {
  using L = RevLay;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  unsigned char* sm = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::SM_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + L::SM_TMEM);
  ScanVec* vecs = reinterpret_cast<ScanVec*>(sm + L::SM_VEC);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh - b * H;
  const int hq = h * Hk / H;
  const int c0 = blockIdx.x * DVT;
  const int N = (T + C - 1) / C;
  // iteration it handles chunk N - 1 - it

  if (tid == 0) {
    for (int i = 0; i < kRevNS; ++i) {
      mbar_init(&bars[R_FULL + i], 1);
      mbar_init(&bars[R_EMPTY + i], 1);
    }
    for (int i = 0; i < kRevNR; ++i) {
      mbar_init(&bars[R_ZFULL + i], 1);
      mbar_init(&bars[R_ZEMPTY + i], 1);
    }
    for (int i = 0; i < NV; ++i) {
      mbar_init(&bars[R_VFULL + i], 1);
      mbar_init(&bars[R_VEMPTY + i], 8);
    }
    mbar_init(&bars[R_D1], 1);
    mbar_init(&bars[R_X], 4);
    mbar_init(&bars[R_E], 4);
    mbar_init(&bars[R_D3], 1);
    mbar_init(&bars[R_S], 8);
    mbar_init(&bars[R_D1FREE + 0], 4);
    mbar_init(&bars[R_D1FREE + 1], 4);
    mbar_init(&bars[R_DONE], 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, ST_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sbase = smem_u32(sm);

  if (warp == 0) {
    // ---- K, Q and this CTA's dO columns of each chunk (TMA) ----
    if (elect_one()) {
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmO);
      if (dhsb) prefetch_tmap(&tmV);
      int issued = 0;
      for (int it = 0; it < N; ++it) {
        const int n = N - 1 - it, s = it % kRevNS;
        if (it >= kRevNS && !mbar_wait(&bars[R_EMPTY + s], (uint32_t)((it / kRevNS) - 1) & 1u))
          break;
        unsigned char* kq = sm + L::SM_KQ + s * 32768;
        uint64_t* fb = &bars[R_FULL + s];
        mbar_arrive_expect_tx(fb, dhsb ? 32768 + 16384 : 32768 + 8192);
        for (int kb = 0; kb < 2; ++kb) {
          tma_load_4d(kq + kb * 16384, &tmK, 64 * kb, hq, n * C, b, fb);
          tma_load_4d(kq + kb * 16384 + 8192, &tmQ, 64 * kb, hq, n * C, b, fb);
        }
        tma_load_4d(sm + L::SM_DO + s * 8192, &tmO, c0, h, n * C, b, fb);
        if (dhsb) tma_load_4d(sm + L::SM_V + s * 8192, &tmV, c0, h, n * C, b, fb);
        issued = it + 1;
      }
      for (int it = issued > kRevNS ? issued - kRevNS : 0; it < issued; ++it)
        mbar_wait(&bars[R_FULL + it % kRevNS], (uint32_t)(it / kRevNS) & 1u);
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (elect_one()) {
      bool ok = true;
      for (int it = 0; it < N && ok; ++it) {
        const int s = it % kRevNS, r = it % kRevNR, buf = it & 1;
        const uint32_t kq = sbase + L::SM_KQ + s * 32768;
        const uint32_t zt = sbase + L::SM_Z + r * kRevTile;
        ok = mbar_wait(&bars[R_ZFULL + r], (uint32_t)(it / kRevNR) & 1u) &&
             mbar_wait(&bars[R_FULL + s], (uint32_t)(it / kRevNS) & 1u) &&
             (it < 2 || mbar_wait(&bars[R_D1FREE + buf], (uint32_t)((it - 2) >> 1) & 1u));
        if (!ok) break;
        tc_fence_after();
        // D1 = PT^T dO first (Y, independent of R): A = PT^T (M = tokens i) read
        // MN-major from the PT rows [j][i]; B = dO [j][64 columns], MN-major;
        // K-dim = the chunk's 64 tokens j.  The second 64-row M block of every
        // A here (LBO ahead, in shared memory) only feeds rows 64-127 of D1,
        // which are not read.
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t a = umma_desc(zt + 16384 + k * 2048, 8192, 1024, SW128);
          const uint64_t bd = umma_desc(sbase + L::SM_DO + s * 8192 + k * 2048, 8192, 1024, SW128);
          mma_bf16(tmem + ST_D1 + (uint32_t)buf * 64, a, bd, IDESC_MM, k > 0);
        }
        ok = mbar_wait(&bars[R_S], (uint32_t)it & 1u);
        if (!ok) break;
        tc_fence_after();
        // D1 += Z R: A = Z (M = tokens) read MN-major from the Z tile [key][token],
        // B = the gradient tile, K-dim = dk in 8 steps
#pragma unroll
        for (int k = 0; k < DK / 16; ++k) {
          const uint64_t a = umma_desc(zt + k * 2048, 8192, 1024, SW128);
          const uint64_t bd = umma_desc(sbase + L::SM_S + k * 2048, 16384, 1024, SW128);
          mma_bf16(tmem + ST_D1 + (uint32_t)buf * 64, a, bd, IDESC_MM, 1u);
        }
        mma_commit(&bars[R_D1]);
        if (dhsb) {
          // the bf16 gradient leaving chunk N - 1 - it, as the tile D1 just read
          bulk_s2g(dhsb + (((size_t)b * N + (N - 1 - it)) * H + h) * kHandoffDhSlot +
                       blockIdx.x * 16384,
                   sm + L::SM_S, 16384);
          bulk_commit();
        }
        // D3 = Q^T (e dO) first (A = Q^T, MN-major, M = dk in two 64-wide
        // blocks 16 KB apart), then + K^T X once X is formed
        ok = mbar_wait(&bars[R_E], (uint32_t)it & 1u);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t a = umma_desc(kq + 8192 + k * 2048, 16384, 1024, SW128);
          const uint64_t bd = umma_desc(sbase + L::SM_E + k * 2048, 8192, 1024, SW128);
          mma_bf16(tmem + ST_D3, a, bd, IDESC_MM, k > 0);
        }
        ok = mbar_wait(&bars[R_X], (uint32_t)it & 1u);
        if (!ok) break;
        // the gradient tile is rewritten once D3 completes: its copy has read it
        if (dhsb) bulk_wait_read<0>();
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t a = umma_desc(kq + k * 2048, 16384, 1024, SW128);
          const uint64_t bd = umma_desc(sbase + L::SM_X + k * 2048, 8192, 1024, SW128);
          mma_bf16(tmem + ST_D3, a, bd, IDESC_MM, 1u);
        }
        mma_commit(&bars[R_D3]);
        mma_commit(&bars[R_EMPTY + s]);
        mma_commit(&bars[R_ZEMPTY + r]);
      }
      mma_commit(&bars[R_DONE]);
      mbar_wait(&bars[R_DONE], 0);
      if (dhsb) bulk_wait<0>();
    }
  } else if (warp == 2) {
    // ---- gate warp: beta, e^G and e^{G_C} of each chunk, NV - 1 chunks ahead ----
    const size_t gb = (size_t)b * T * H + h;
    for (int it = 0; it < N; ++it) {
      const int n = N - 1 - it, v = it % NV;
      const int t = n * C + 2 * lane;
      const float g0 = t < T ? ldg_f32(g + gb + (size_t)t * H) : 0.f;
      const float g1 = t + 1 < T ? ldg_f32(g + gb + (size_t)(t + 1) * H) : 0.f;
      const float b0 = t < T ? ldg_f32(beta + gb + (size_t)t * H) : 0.f;
      const float b1 = t + 1 < T ? ldg_f32(beta + gb + (size_t)(t + 1) * H) : 0.f;
      if (it >= NV && !mbar_wait(&bars[R_VEMPTY + v], (uint32_t)((it / NV) - 1) & 1u)) break;
      ScanVec& vb = vecs[v];
      const float pair = g0 + g1;
      float incl = pair;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += y;
      }
      vb.beta[2 * lane] = b0;
      vb.beta[2 * lane + 1] = b1;
      vb.eG[2 * lane] = gate_exp(incl - pair + g0);
      vb.eG[2 * lane + 1] = gate_exp(incl);
      if (lane == 31) vb.eGC = gate_exp(incl);
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[R_VFULL + v]);
    }
  } else if (warp == 3) {
    // ---- [Z | PT] tiles (bulk copies of the first 24 KB of each slot) ----
    if (elect_one()) {
      const unsigned char* src = tiles + (size_t)bh * N * kTileBytesBwd;
      int issued = 0;
      for (int it = 0; it < N; ++it) {
        const int n = N - 1 - it, r = it % kRevNR;
        if (it >= kRevNR && !mbar_wait(&bars[R_ZEMPTY + r], (uint32_t)((it / kRevNR) - 1) & 1u))
          break;
        mbar_arrive_expect_tx(&bars[R_ZFULL + r], kRevTile);
        bulk_g2s(sm + L::SM_Z + r * kRevTile, src + (size_t)n * kTileBytesBwd, kRevTile,
                 &bars[R_ZFULL + r]);
        issued = it + 1;
      }
      for (int it = issued > kRevNR ? issued - kRevNR : 0; it < issued; ++it)
        mbar_wait(&bars[R_ZFULL + it % kRevNR], (uint32_t)(it / kRevNR) & 1u);
    }
  } else {
    // ---- epilogue warps: quarter wq of the TMEM lanes, 32 of the 64 columns ----
    const int wq = warp & 3;
    const int cb = 32 * ((warp - 4) >> 2);  // column offset within the tile
    const int r = wq * 32 + lane;           // TMEM lane: key row, or token row
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    unsigned char* Stile = sm + L::SM_S;
    // store staging, 4 KB per block: the gradient block of epilogue warp e at
    // slot e, the dX block of the warps on lanes 0-63 at slots 8-11
    const int ew = warp - 4, xw = wq + 2 * (cb >> 5);
    unsigned char* stg_r = sm + L::SM_STG + ew * 4096;
    unsigned char* stg_x = sm + L::SM_STG + (8 + xw) * 4096;
    auto stage_store = [&](unsigned char* stg, const float (&vals)[32], const CUtensorMap* map,
                           int x, int y) {
      if (lane == 0) bulk_wait_read<0>();
      __syncwarp();
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8)
        *reinterpret_cast<float4*>(stg + sw128(lane, c8)) =
            make_float4(vals[4 * c8], vals[4 * c8 + 1], vals[4 * c8 + 2], vals[4 * c8 + 3]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(map, x, y, stg);
        bulk_commit();
      }
    };
    float R[32];
    {
      const float* src = dhT ? dhT + ((size_t)bh * DK + r) * dv + c0 + cb : nullptr;
#pragma unroll
      for (int c = 0; c < 32; c += 4) {
        const float4 x = src ? *reinterpret_cast<const float4*>(src + c)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
        R[c] = x.x; R[c + 1] = x.y; R[c + 2] = x.z; R[c + 3] = x.w;
      }
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8)
        *reinterpret_cast<uint4*>(Stile + sw128(r, cb / 8 + c8)) = pack_bf16x8(R + 8 * c8);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[R_S]);
      // the gradient leaving the last chunk
      if (!dhsb)
        stage_store(stg_r, R, &tmDHS, c0 + cb,
                    (int)((((size_t)b * N + N - 1) * H + h) * DK) + wq * 32);
    }
    bool ok = true;
    for (int it = 0; it < N && ok; ++it) {
      const int n = N - 1 - it, s = it % kRevNS, v = it % NV, buf = it & 1;
      const ScanVec& vb = vecs[v];
      const size_t slot = ((size_t)b * N + n) * H + h;   // workspace slot of (chunk, head)
      ok = mbar_wait(&bars[R_VFULL + v], (uint32_t)(it / NV) & 1u);
      if (!ok) break;
      if (wq < 2) {
        // ---- dX = D1 = PT^T dO + Z R, token row r; X = -beta e dX ----
        const bool in = n * C + r < T;
        uint4 vrow[4];   // (hand-off) this row's 32 columns of v, read ahead of D1
        if (dhsb) {
          ok = mbar_wait(&bars[R_FULL + s], (uint32_t)(it / kRevNS) & 1u);
          if (!ok) break;
          const unsigned char* Vt = sm + L::SM_V + s * 8192;
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8)
            vrow[c8] = *reinterpret_cast<const uint4*>(Vt + sw128(r, cb / 8 + c8));
        }
        const float sc = -vb.beta[r] * vb.eG[r];
        ok = mbar_wait(&bars[R_D1], (uint32_t)it & 1u);
        if (!ok) break;
        tc_fence_after();
        float y[32];
        tmem_ld32(tmem + ST_D1 + (uint32_t)buf * 64 + (uint32_t)cb + lane_off, y);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[R_D1FREE + buf]);
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          float x[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) x[e] = sc * y[8 * c8 + e];
          *reinterpret_cast<uint4*>(sm + L::SM_X + sw128(r, cb / 8 + c8)) = pack_bf16x8(x);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[R_X]);
        // dX, after the arrival (which gates the chain); rows past T hold
        // dX = 0 (their columns of PT and their rows of Z are zero)
        if (dhsb) {
          // dV = beta dX, the row's partial rowsum(dX o v), dX as bf16
          const float bi = vb.beta[r];
          float xv = 0.f;
          __nv_bfloat16* dst = dvo + (((size_t)b * T + (size_t)n * C + r) * H + h) * dv + c0 + cb;
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            float vv[8], o8[8];
            unpack_bf16x8(vrow[c8], vv);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              xv = fmaf(y[8 * c8 + e], vv[e], xv);
              o8[e] = bi * y[8 * c8 + e];
            }
            if (in) *reinterpret_cast<uint4*>(dst + 8 * c8) = pack_bf16x8(o8);
          }
          reinterpret_cast<float*>(dhsb + slot * kHandoffDhSlot + 32768)[r * 4 + (c0 + cb) / 32] = xv;
          // dX as bf16 into this warp's staging; the proxy fence that the
          // gradient tile's epilogue below issues anyway covers it, and the
          // tensor store goes out after that epilogue's arrival
          if (lane == 0) bulk_wait_read<0>();
          __syncwarp();
          uint4 pk[4];
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) pk[c8] = pack_bf16x8(y + 8 * c8);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int jc = (c + (lane >> 1)) & 3;   // bank-spread order (as stage_store_bf16)
            const uint4 w = jc == 0 ? pk[0] : jc == 1 ? pk[1] : jc == 2 ? pk[2] : pk[3];
            *reinterpret_cast<uint4*>(stg_x + lane * 64 + jc * 16) = w;
          }
        } else {
          stage_store(stg_x, y, &tmYX, c0 + cb, (int)(slot * C) + wq * 32);
        }
      } else {
        // ---- e dO, token row r - 64, the B operand of Q^T (e dO) ----
        ok = mbar_wait(&bars[R_FULL + s], (uint32_t)(it / kRevNS) & 1u);
        if (!ok) break;
        const int i = r - 64;
        const float ei = vb.eG[i];
        const unsigned char* dOt = sm + L::SM_DO + s * 8192;
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          float x[8];
          unpack_bf16x8(*reinterpret_cast<const uint4*>(dOt + sw128(i, cb / 8 + c8)), x);
#pragma unroll
          for (int e = 0; e < 8; ++e) x[e] *= ei;
          *reinterpret_cast<uint4*>(sm + L::SM_E + sw128(i, cb / 8 + c8)) = pack_bf16x8(x);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[R_E]);
      }
      // ---- R <- e^{G_C} R + D3, key row r ----
      ok = mbar_wait(&bars[R_D3], (uint32_t)it & 1u);
      if (!ok) break;
      tc_fence_after();
      {
        float d3[32];
        tmem_ld32(tmem + ST_D3 + (uint32_t)cb + lane_off, d3);
        const float egc = vb.eGC;
#pragma unroll
        for (int e = 0; e < 32; ++e) R[e] = fmaf(egc, R[e], d3[e]);
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8)
          *reinterpret_cast<uint4*>(Stile + sw128(r, cb / 8 + c8)) = pack_bf16x8(R + 8 * c8);
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[R_S]);
        if (!dhsb && n > 0)   // the gradient leaving chunk n - 1
          stage_store(stg_r, R, &tmDHS, c0 + cb, (int)((slot - H) * DK) + wq * 32);
        if (dhsb && wq < 2 && lane == 0) {   // this chunk's dX rows, staged above
          tma_store_2d(&tmYX, c0 + cb, (int)(slot * C) + wq * 32, stg_x);
          bulk_commit();
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[R_VEMPTY + v]);
    }
    if (ok && dh0) {
      float* dst = dh0 + ((size_t)bh * DK + r) * dv + c0 + cb;
#pragma unroll
      for (int c = 0; c < 32; c += 4)
        *reinterpret_cast<float4*>(dst + c) = make_float4(R[c], R[c + 1], R[c + 2], R[c + 3]);
    }
    if (lane == 0) bulk_wait<0>();   // every tensor store done before exit
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, ST_COLS);
  }
}

}  // namespace

GDN_DEVICE_ERROR_ACCESSOR(device_error_chunk_scan)

int chunk_scan_binary_version() {
  cudaFuncAttributes fa;
  if (cudaFuncGetAttributes(&fa, chunk_scan_kernel<false>) != cudaSuccess) return -1;
  return fa.binaryVersion;
}

bool chunk_scan_shape_ok(const ChunkArgs& a) {
  return a.dtype == kBF16 && a.semantics == kExact && a.dk == DK && a.dv % DVT == 0 &&
         a.T > 0 && !a.cu_seqlens && (long long)a.B * a.H <= 65535;
}

bool chunk_scan_supported(const ChunkArgs& a) {
  return chunk_scan_shape_ok(a) && encode_fn() != nullptr;
}

size_t chunk_scan_workspace_bytes(int B, int T, int H) {
  if (B <= 0 || T <= 0 || H <= 0) return 0;
  const size_t N = ((size_t)T + C - 1) / C;
  return (size_t)B * H * N * kTileBytes;
}

size_t chunk_scan_bwd_tiles_bytes(int B, int T, int H) {
  if (B <= 0 || T <= 0 || H <= 0) return 0;
  const size_t N = ((size_t)T + C - 1) / C;
  return (size_t)B * H * N * kTileBytesBwd;
}

namespace {

// TMA maps of q and k (dk = 128) over the dense rows.
bool qk_maps(const ChunkArgs& a, CUtensorMap* mk, CUtensorMap* mq) {
  return make_bf16_map_4d(mk, a.k, a.B, a.T, a.Hk, DK) &&
         make_bf16_map_4d(mq, a.q, a.B, a.T, a.Hk, DK);
}

bool workspace_ok(const ChunkArgs& a) {
  return a.workspace && a.ws_bytes >= chunk_scan_workspace_bytes(a.B, a.T, a.H) &&
         (reinterpret_cast<uintptr_t>(a.workspace) & 15u) == 0;
}

}  // namespace

template <bool kT>
cudaError_t launch_prepare_t(const ChunkArgs& a, cudaStream_t st) {
  CUtensorMap mk, mq;
  if (!qk_maps(a, &mk, &mq)) return cudaErrorInvalidValue;
  static std::atomic<int> prep_slot[kMaxDevices] = {};
  cudaError_t e = ensure_smem(chunk_prep_kernel<kT>, PrepLay::SMEM_BYTES, prep_slot);
  if (e != cudaSuccess) return e;
  const int N = (a.T + C - 1) / C;
  const long long items = (long long)a.B * a.H * N;
  const int prep_ctas = (int)(items < 2LL * device_sm_count() ? items : 2LL * device_sm_count());
  chunk_prep_kernel<kT><<<prep_ctas, kPrepThreads, PrepLay::SMEM_BYTES, st>>>(
      mk, mq, a.g, a.beta, static_cast<unsigned char*>(a.workspace), a.T, a.H, a.Hk,
      a.B * a.H, N);
  return cudaGetLastError();
}

cudaError_t launch_chunk_prepare(const ChunkArgs& a, cudaStream_t st) {
  if ((long long)a.B * a.H == 0 || a.T == 0) return cudaSuccess;
  if (!chunk_scan_supported(a) || !workspace_ok(a)) return cudaErrorInvalidValue;
  return launch_prepare_t<false>(a, st);
}

cudaError_t launch_chunk_prepare_bwd(const ChunkArgs& a, cudaStream_t st) {
  if ((long long)a.B * a.H == 0 || a.T == 0) return cudaSuccess;
  if (!chunk_scan_supported(a) || !a.workspace ||
      a.ws_bytes < chunk_scan_bwd_tiles_bytes(a.B, a.T, a.H) ||
      (reinterpret_cast<uintptr_t>(a.workspace) & 15u) != 0)
    return cudaErrorInvalidValue;
  return launch_prepare_t<true>(a, st);
}

cudaError_t launch_chunk_scan_prepared(const ChunkArgs& a, bool transition, cudaStream_t st) {
  if ((long long)a.B * a.H == 0 || a.T == 0) return cudaSuccess;
  if (!chunk_scan_supported(a) || !workspace_ok(a)) return cudaErrorInvalidValue;
  CUtensorMap mk, mq, mv;
  if (!qk_maps(a, &mk, &mq) || !make_bf16_map_4d(&mv, a.v, a.B, a.T, a.H, a.dv))
    return cudaErrorInvalidValue;
  static std::atomic<int> scan_slot[kMaxDevices] = {};
  cudaError_t e = ensure_smem(chunk_scan_kernel<false>, ScanLay::SMEM_BYTES, scan_slot);
  if (e != cudaSuccess) return e;
  const int ds = a.dv + (transition ? DK : 0);
  // Launched with programmatic stream serialization: when the preparation runs
  // right before on the stream, the scan's set-up overlaps the preparation's
  // last wave, and its reads of the workspace wait for the whole preparation
  // grid (griddep_wait); otherwise this is an ordinary launch.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ds / DVT, a.B * a.H);
  cfg.blockDim = dim3(kScanThreads);
  cfg.dynamicSmemBytes = ScanLay::SMEM_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, chunk_scan_kernel<false>, mk, mq, mv, a.g, a.beta,
                         static_cast<const unsigned char*>(a.workspace), a.h0,
                         static_cast<__nv_bfloat16*>(a.o), a.hT, a.T, a.H, a.Hk, a.dv, ds,
                         mk, mk,   // (the state maps are read in the backward mode only)
                         static_cast<unsigned char*>(nullptr));
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_chunk_scan_bwd(const ChunkArgs& a, float* hs, float* vp, bool hs_tiles,
                                  cudaStream_t st) {
  if ((long long)a.B * a.H == 0 || a.T == 0) return cudaSuccess;
  if (!chunk_scan_supported(a) || a.dv != 128 || !a.workspace || !hs || !vp ||
      a.ws_bytes < chunk_scan_bwd_tiles_bytes(a.B, a.T, a.H))
    return cudaErrorInvalidValue;
  CUtensorMap mk, mq, mv, mhs, mvp;
  const long long slots = (long long)a.B * ((a.T + C - 1) / C) * a.H;
  // (with hs_tiles the states go out by bulk copies: no fp32 map over hs, whose
  // region then holds only the bf16 tiles)
  if (!qk_maps(a, &mk, &mq) || !make_bf16_map_4d(&mv, a.v, a.B, a.T, a.H, a.dv) ||
      !(hs_tiles || make_f32_map_2d(&mhs, hs, slots * DK, a.dv)) ||
      !(hs_tiles ? make_bf16_map_2d(&mvp, vp, slots * C, a.dv, false)
                 : make_f32_map_2d(&mvp, vp, slots * C, a.dv)))
    return cudaErrorInvalidValue;
  if (hs_tiles) mhs = mvp;   // (not read)
  static std::atomic<int> slot[kMaxDevices] = {};
  cudaError_t e = ensure_smem(chunk_scan_kernel<true>, ScanLay::SMEM_BYTES, slot);
  if (e != cudaSuccess) return e;
  chunk_scan_kernel<true><<<dim3(a.dv / DVT, a.B * a.H), kScanThreads, ScanLay::SMEM_BYTES, st>>>(
      mk, mq, mv, a.g, a.beta, static_cast<const unsigned char*>(a.workspace), a.h0, nullptr,
      nullptr, a.T, a.H, a.Hk, a.dv, a.dv, mhs, mvp,
      hs_tiles ? reinterpret_cast<unsigned char*>(hs) : nullptr);
  return cudaGetLastError();
}

cudaError_t launch_chunk_scan_rev(const ChunkArgs& a, const void* dO, const float* dhT,
                                  float* dh0, float* yx, float* dhs, void* dxb, void* dvo,
                                  cudaStream_t st) {
  if ((long long)a.B * a.H == 0 || a.T == 0) return cudaSuccess;
  const bool hand = dxb != nullptr;
  if (!chunk_scan_supported(a) || a.dv != 128 || !a.workspace || !dO || !yx || !dhs ||
      a.ws_bytes < chunk_scan_bwd_tiles_bytes(a.B, a.T, a.H) || (hand && (!dvo || !a.v)))
    return cudaErrorInvalidValue;
  CUtensorMap mk, mq, mo, myx, mdhs, mv;
  const long long slots = (long long)a.B * ((a.T + C - 1) / C) * a.H;
  // (with the hand-off the gradients go out by bulk copies: no fp32 map over
  // dhs, whose region then holds only the bf16 tiles and row partials)
  if (!qk_maps(a, &mk, &mq) || !make_bf16_map_4d(&mo, dO, a.B, a.T, a.H, a.dv) ||
      !(hand || make_f32_map_2d(&mdhs, dhs, slots * DK, a.dv)) ||
      !(hand ? make_bf16_map_2d(&myx, dxb, slots * C, a.dv, false) &&
                   make_bf16_map_4d(&mv, a.v, a.B, a.T, a.H, a.dv)
             : make_f32_map_2d(&myx, yx, slots * C, a.dv)))
    return cudaErrorInvalidValue;
  if (hand) mdhs = mo;   // (not read)
  else mv = mo;
  static std::atomic<int> slot[kMaxDevices] = {};
  cudaError_t e = ensure_smem(chunk_scan_rev_kernel, RevLay::SMEM_BYTES, slot);
  if (e != cudaSuccess) return e;
  chunk_scan_rev_kernel<<<dim3(a.dv / DVT, a.B * a.H), kScanThreads, RevLay::SMEM_BYTES, st>>>(
      mk, mq, mo, a.g, a.beta, static_cast<const unsigned char*>(a.workspace), dhT, dh0, myx,
      mdhs, hand ? reinterpret_cast<unsigned char*>(dhs) : nullptr, mv,
      static_cast<__nv_bfloat16*>(dvo), a.T, a.H, a.Hk, a.dv);
  return cudaGetLastError();
}

cudaError_t launch_chunk_scan(const ChunkArgs& a, cudaStream_t st) {
  cudaError_t e = launch_chunk_prepare(a, st);
  if (e != cudaSuccess) return e;
  return launch_chunk_scan_prepared(a, false, st);
}

}  // namespace gdn
