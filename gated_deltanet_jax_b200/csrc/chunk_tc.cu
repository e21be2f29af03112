// Chunked gated delta-rule forward on 5th-generation tensor cores, sm_100a.
//
// Replaces chunk_gated_delta_rule_fwd (ops.py:299-346) for bf16 inputs with
// dk = 128 or 256, dv a multiple of 64 (exact semantics, in chunks of 64
// whatever the requested chunk length).  Every matrix product is a tcgen05.mma
// (bf16 operands in shared memory, fp32 accumulators in tensor memory) fed by
// TMA tile loads; the state stays on chip for the whole sequence.
//
// dk = 256 (the head_dim of the reference's default configuration) uses the
// same roles and products with twice the key steps: one K/Q stage of 64 KB
// instead of two (so the next chunk's tiles load only once this one's are
// released), the state increment K^T V'' as two M = 128 products (TMEM
// columns 320 and 448), and two state rows (r, r + 128) per chain thread.
// Only the unpaired form exists for it.
//
// One CTA owns one (b, h) and a tile of 64 state columns, and walks the
// chunks in order.  Per chunk n (C = 64 tokens, in-chunk cumulative gate G):
//
//   prep (independent of the state; runs one chunk ahead):
//     D_pre = [K;Q] K^T                      (M=128: rows K K^T, then Q K^T)
//     A = tril_{-1}(beta_i e^{G_i-G_j} K K^T),  P = tril_0(e^{G_i-G_j} Q K^T)
//     T = (I + A)^{-1}                       (16x16 diagonal blocks by fp32 substitution,
//                                             off-diagonal blocks on tf32 warp MMAs)
//     tile TP = [T; P] (bf16, 128 x 64)
//   chain (sequential over chunks, state S [128 x 64] fp32 in registers):
//     D1 = [K;Q] S_bf16                      rows 0-63: K S, rows 64-127: Q S
//     X  = beta (V - e^G (K S))              -> bf16 tile
//     D2 = [T;P] X                           rows 0-63: V' = T X
//     V'' = e^{G_C - G} V'                   -> bf16 tiles V'' and V'
//     D3 = K^T V''                           (the state increment, M = dk)
//     D4 = [T;P] V'                          rows 64-127: P V'
//     S <- e^{G_C} S + D3                    -> bf16 tile for the next chunk
//     O = e^G (Q S) + P V'                   (rows 64-127 of D1 and D4)
//
// Warp roles (512 threads): warp 0 issues TMA loads, warp 1 the chain MMAs
// and owns the tensor memory, warp 2 the prep MMAs, warp 3 computes the gate
// vectors two chunks ahead; warps 4-11 do the prep math (two warps per TMEM
// lane quarter, one per 32 columns), warps 12-15 the chain epilogues.  A warp
// reads only its own quarter of the 128 TMEM lanes, so row r of every M=128
// accumulator belongs to thread r of a warpgroup.  All hand-offs are
// mbarriers; every wait is bounded.
//
// Layer form (kLayer, dk = dv = 128, the two column tiles of a row as one
// cluster of two CTAs, with or without shared preparation): the GatedDeltaNet
// layer's work on either side of the op in the same kernel (model.py:136-139,
// :47-53).  The gate warp forms beta = sigmoid(b) and g = -exp(A_log[h])
// softplus(a + dt_bias[h]) from the raw projections.  The output epilogue sums
// the squares of its 64 fp32 columns of each row, stages the row as bf16 in
// shared memory, releases TMEM, and sends the partial sum into the other CTA's
// shared memory (one st.async per row, completing on its barrier).  The row is
// finished at the start of the next chunk, when the other CTA's sum has
// arrived: y = o rsqrt(mean(o^2) + eps) w silu(gate) replaces o.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "chunk_common.cuh"
#include "gdn_common.cuh"
#include "gdn_internal.h"
#include "ptx.cuh"

namespace gdn {

namespace {

constexpr int DVT = 64;
constexpr int kThreads = 512;
// Register split (per thread): the kernel is compiled for, and launched with,
// kLaunchRegs; warpgroup 0 (producer, MMA issuers, gate) gives registers to the
// chain warpgroup.  4 x 128 threads x (56 + 128 + 128 + 200) = 512 x 128.
constexpr int kLaunchRegs = 128;
constexpr int kRegsRoles = 56, kRegsPrep = 128, kRegsChain = 200;
static_assert(kRegsRoles + 2 * kRegsPrep + kRegsChain == 4 * kLaunchRegs, "register split");
constexpr int NTP = 3;   // depth of the T/P tile and gate-vector rings
constexpr int NBAR = 40;
// Layer form: ring of the other tile's row sums of squares.  A row is finished
// one chunk after its products (its sum is read at the start of the next
// chunk).  A CTA's chain runs at most NTP chunks ahead of the other's: with
// shared preparation, because a T/P slot is refilled only after both chains
// released it; without, because finishing row m waits for the other CTA's sum
// of chunk m.  So NTP + 1 slots keep a slot from being rewritten before it
// was read.
constexpr int NSS = NTP + 1;

// Shared-memory byte offsets from a 1024-byte aligned base, for key width DK
// (128 or 256).  K and Q of a chunk sit in DK / 64 blocks of [128 rows][128 B]
// (rows 0-63 K, 64-127 Q, 64 key dimensions each).  DK = 256 keeps one such
// stage (64 KB) instead of two, and has no layer-form buffers, to stay within
// 227 KB.
template <int DK>
struct Lay {
  static constexpr int NSTAGE = DK == 128 ? 2 : 1;
  static constexpr int KQ_STAGE = DK / 64 * 16384;
  static constexpr int SM_KQ = 0;                          // NSTAGE x KQ_STAGE
  static constexpr int SM_V = SM_KQ + NSTAGE * KQ_STAGE;   // NSTAGE x [64 rows][128 B]
  static constexpr int SM_S = SM_V + NSTAGE * 8192;        // [DK rows][128 B]
  static constexpr int SM_X = SM_S + DK * 128;             // [64 rows (token)][128 B]
  static constexpr int SM_VPP = SM_X + 8192;               // V'' = e^{G_C-G} V'
  static constexpr int SM_VP = SM_VPP + 8192;              // V'
  static constexpr int SM_TP = SM_VP + 8192;               // NTP x [128 rows][128 B]: T, P
  static constexpr int SM_AF = SM_TP + NTP * 16384;        // fp32 A [64][LDF]
  static constexpr int SM_TF = SM_AF + 64 * LDF * 4;       // fp32 T [64][LDF]
  static constexpr int SM_VEC = SM_TF + 64 * LDF * 4;      // NTP x VecBuf
  static constexpr int SM_BAR = SM_VEC + NTP * (int)sizeof(VecBuf);
  static constexpr int SM_TMEM = SM_BAR + NBAR * 8;
  static constexpr bool kHasLayer = DK == 128;
  static constexpr int SM_SS = SM_TMEM + 16;               // layer form: NSS x [64] row sums
  static constexpr int SM_W = SM_SS + (kHasLayer ? NSS * 64 * 4 : 0);  // layer: norm weight
  static constexpr int SM_OB = SM_W + (kHasLayer ? DVT * 4 : 0);       // layer: bf16 rows
  static constexpr int SM_TOTAL = SM_OB + (kHasLayer ? 8192 : 0);
  static constexpr int SMEM_BYTES = SM_TOTAL + 1024;       // + alignment slack
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
};

// barrier indices
enum {
  B_FULL = 0,        // [NSTAGE] TMA stage loaded
  B_EMPTY = 2,       // [NSTAGE] stage consumed by the MMAs
  B_PRE_FULL = 4,    // [2] D_pre ready
  B_PRE_EMPTY = 6,   // [2] D_pre read by prep
  B_TP_READY = 8,    // [NTP] T/P tile of a chunk in this CTA's ring (made here or copied in)
  B_TP_EMPTY = 11,   // [NTP] every chain of the pair is done with a chunk's tile
  B_VEC_FULL = 14,   // [NTP] gate vectors of a chunk ready
  B_VEC_EMPTY = 17,  // [NTP] this CTA's chain is done with a chunk's gate vectors
  B_D1 = 20, B_D2 = 21, B_D3 = 22, B_D4 = 23, B_D4_EMPTY = 24,
  B_X_READY = 25, B_VPP_READY = 26, B_S_READY = 27, B_CHAIN_DONE = 28,
  B_SS = 29,         // [NSS] layer form: the other tile's row sums of squares of a chunk arrived
};
static_assert(B_SS + NSS <= NBAR, "barriers");

// TMEM columns
constexpr uint32_t TM_PRE = 0;    // 2 x 64
constexpr uint32_t TM_D1 = 128;   // 2 x 64
constexpr uint32_t TM_D2 = 256;
constexpr uint32_t TM_D3 = 320;   // DK = 256: a second M = 128 half at TM_D3 + 128
constexpr uint32_t TM_D4 = 384;
constexpr uint32_t TM_COLS = 512;


// silu(z) = z sigmoid(z) = z (1 + tanh(z / 2)) / 2, on the PTX instruction
// tanh.approx.f32 (documented maximum relative error about 2^-11, one
// special-function op where e^-z and a reciprocal take two): its error stays
// far below the bf16 rounding of the layer output it scales.
__device__ __forceinline__ float silu_fast(float z) {
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.5f * z));
  const float hz = 0.5f * z;
  return fmaf(hz, t, hz);
}

// Bounded wait by a single thread (the elected lane of a one-thread role).
__device__ __forceinline__ bool wait_bar(uint64_t* bars, int idx, uint32_t parity) {
  return mbar_wait(&bars[idx], parity);
}

// Waits on barriers that the other CTA of a pair also arrives on.
template <bool kPair>
__device__ __forceinline__ bool wait_shared_bar(uint64_t* bars, int idx, uint32_t parity) {
  return kPair ? mbar_wait_cluster(&bars[idx], parity) : mbar_wait(&bars[idx], parity);
}

// kPair: the grid is launched in clusters of two CTAs, the two 64-column
// tiles of one (b, h).  Each prepares the T/P tile of every other chunk (rank
// r: chunks n with n % 2 == r) and copies it into the other CTA's ring, so
// the state-independent preparation is done once per (b, h) rather than once
// per column tile.
// kLayer (dv = 128 only): g and beta hold the raw a_proj / b_proj outputs,
// and o receives the gated RMSNorm of the output (la).  The two column tiles
// of a row always run as a cluster of two CTAs, which exchange the rows'
// partial sums of squares; without kPair each still prepares every chunk (the
// compact form, for high occupancy).
// kGates (implied by kLayer): g and beta hold the raw a_proj / b_proj outputs
// and the gate warp forms g and beta from them (la.A_log, la.dt_bias); without
// kLayer the output is the op's o, for a separate gated RMSNorm (the layer at
// head dims other than dk = dv = 128).
// h0 and hT may be the same array (in-place state): each CTA reads its tile of
// h0 before the loop and writes the same tile of hT after it.
template <int DK, bool kPair, bool kLayer, bool kGates = kLayer>
__global__ void __launch_bounds__(kThreads, 1)
chunk_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmQ,
                const __grid_constant__ CUtensorMap tmV, const float* __restrict__ g,
                const float* __restrict__ beta, const float* h0,
                __nv_bfloat16* __restrict__ o, float* hT,
                const int* __restrict__ cu_seqlens, int T, int H, int Hk, int dv,
                const LayerArgs la) {
  constexpr bool kCluster = kPair || kLayer;  // launched in clusters of two CTAs
  static_assert(DK == 128 || (DK == 256 && !kPair && !kLayer), "key width");
  static_assert(kGates || !kLayer, "the layer form forms its own gates");
  using L = Lay<DK>;
  constexpr int NSTAGE = L::NSTAGE, KQ_STAGE = L::KQ_STAGE;
  constexpr int SM_KQ = L::SM_KQ, SM_V = L::SM_V, SM_S = L::SM_S, SM_X = L::SM_X;
  constexpr int SM_VPP = L::SM_VPP, SM_VP = L::SM_VP, SM_TP = L::SM_TP, SM_AF = L::SM_AF;
  constexpr int SM_TF = L::SM_TF, SM_VEC = L::SM_VEC, SM_BAR = L::SM_BAR, SM_TMEM = L::SM_TMEM;
  constexpr int SM_SS = L::SM_SS, SM_W = L::SM_W, SM_OB = L::SM_OB;
  constexpr int KB = DK / 64;    // 64-dimension key blocks
  constexpr int KSTEPS = DK / 16;  // MMA steps over the key dimension
  constexpr int RG = DK / 128;   // state rows per chain thread (rows r, r + 128)
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // Round up to 1024 bytes by offsetting the shared array itself, so that the
  // compiler keeps every access below in the shared address space.
  const uint32_t raw_addr = smem_u32(smem_raw);
  unsigned char* sm = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + SM_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + SM_TMEM);
  VecBuf* vecs = reinterpret_cast<VecBuf*>(sm + SM_VEC);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.y;
  int b = bh / H;
  const int h = bh - b * H;
  const int hq = h * Hk / H;  // q/k head of this value head (grouped heads)
  // Packed variable-length sequences (cu_seqlens != NULL): blockIdx.y = s * H + h,
  // and sequence s is tokens [cu_seqlens[s], cu_seqlens[s + 1]) of the single
  // row of T tokens (offsets clamped to [0, T], so no access leaves the row).
  // Rows of a chunk past the sequence's end hold the next sequence's tokens (or
  // the zero fill past the row): they get g = beta = 0, which makes their rows
  // of A, X and V' exactly zero, so they reach neither the state nor an output.
  int tok0 = 0, Tn = T;
  if (cu_seqlens) {
    const int a0 = min(max(cu_seqlens[b], 0), T);
    const int a1 = min(max(cu_seqlens[b + 1], a0), T);
    b = 0, tok0 = a0, Tn = a1 - a0;
  }
  const int c0 = blockIdx.x * DVT;
  const int N = (Tn + C - 1) / C;
  // chunks whose T/P tile this CTA prepares: n = rank, rank + step, ...
  const int rank = kPair ? (int)cluster_ctarank() : 0;
  // TMEM read widths of the A/P pass and the chain epilogues.  Paired tiles
  // run one launch per (b, h) pair at low occupancy, where the chain's latency
  // decides: wide, unrolled reads.  Unpaired tiles run at high occupancy, where
  // the instruction fetch of all warps of an SM decides: narrow, rolled reads.
  constexpr int kWP = kPair ? 32 : 16;
  constexpr int kWC = kPair ? 64 : 16;
  const int step = kPair ? 2 : 1;
  // the other CTA of the cluster (pairs: the T/P tiles; layer form: the row sums)
  const uint32_t peer = kCluster ? (cluster_ctarank() ^ 1u) : 0u;

  if (tid == 0) {
    mbar_init(&bars[B_FULL + 0], 1);
    mbar_init(&bars[B_FULL + 1], 1);
    mbar_init(&bars[B_EMPTY + 0], 1);
    mbar_init(&bars[B_EMPTY + 1], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[B_PRE_FULL + i], 1);
      mbar_init(&bars[B_PRE_EMPTY + i], 8);
    }
    for (int i = 0; i < NTP; ++i) {
      mbar_init(&bars[B_TP_READY + i], 1);
      mbar_init(&bars[B_TP_EMPTY + i], kPair ? 8 : 4);
      mbar_init(&bars[B_VEC_FULL + i], 1);
      mbar_init(&bars[B_VEC_EMPTY + i], 4);
    }
    mbar_init(&bars[B_D1], 1);
    mbar_init(&bars[B_D2], 1);
    mbar_init(&bars[B_D3], 1);
    mbar_init(&bars[B_D4], 1);
    mbar_init(&bars[B_D4_EMPTY], 2);
    mbar_init(&bars[B_X_READY], 2);
    mbar_init(&bars[B_VPP_READY], 2);
    mbar_init(&bars[B_S_READY], 4);
    mbar_init(&bars[B_CHAIN_DONE], 1);
    for (int i = 0; i < NSS; ++i) mbar_init(&bars[B_SS + i], 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmV);
  }
  tc_fence_before();
  __syncthreads();
  // the other CTA's barriers are initialised before anything is sent to them
  if (kCluster) cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sbase = smem_u32(sm);

  if (warp < 4) {
    regs_decrease<kRegsRoles>();
    if (warp == 0) {
      // ------------------------------ TMA producer ------------------------------
      if (elect_one()) {
        int issued = 0;
        bool ok = true;
        for (int n = 0; n < N && ok; ++n) {
          const int s = n % NSTAGE;
          if (n >= NSTAGE) ok = wait_bar(bars, B_EMPTY + s, (uint32_t)((n / NSTAGE) - 1) & 1u);
          if (!ok) break;
          unsigned char* kq = sm + SM_KQ + s * KQ_STAGE;
          uint64_t* fb = &bars[B_FULL + s];
          mbar_arrive_expect_tx(fb, KB * 2 * 8192 + 8192);
          const int t0 = tok0 + n * C;
          for (int kb = 0; kb < KB; ++kb) {
            tma_load_4d(kq + kb * 16384, &tmK, 64 * kb, hq, t0, b, fb);
            tma_load_4d(kq + kb * 16384 + 8192, &tmQ, 64 * kb, hq, t0, b, fb);
          }
          tma_load_4d(sm + SM_V + s * 8192, &tmV, c0, h, t0, b, fb);
          issued = n + 1;
        }
        // Let every issued load land before the CTA can exit (bounded).
        for (int n = issued > NSTAGE ? issued - NSTAGE : 0; n < issued; ++n)
          wait_bar(bars, B_FULL + n % NSTAGE, (uint32_t)(n / NSTAGE) & 1u);
      }
    } else if (warp == 1) {
      // ------------------------------ chain MMA issuer ------------------------------
      if (elect_one()) {
        bool ok = true;
        for (int n = 0; n < N && ok; ++n) {
          const int s = n % NSTAGE, tb = n & 1, rb = n % NTP;
          const uint32_t kq = sbase + SM_KQ + s * KQ_STAGE;
          const uint32_t tp = sbase + SM_TP + rb * 16384;
          ok = wait_bar(bars, B_FULL + s, (uint32_t)(n / NSTAGE) & 1u) &&
               wait_bar(bars, B_S_READY, (uint32_t)n & 1u);
          if (!ok) break;
          tc_fence_after();
          // D1 = [K;Q] S   (K-dim = dk: DK / 16 steps of 16)
          const uint32_t d1 = tmem + TM_D1 + (uint32_t)tb * 64;
  #pragma unroll (kPair ? 8 : 1)
          for (int k = 0; k < KSTEPS; ++k) {
            const uint64_t a = umma_desc(kq + (k >> 2) * 16384 + (k & 3) * 32, 16, 1024, SW128);
            const uint64_t bd = umma_desc(sbase + SM_S + k * 2048, 16384, 1024, SW128);
            mma_bf16(d1, a, bd, IDESC_KM, k > 0);
          }
          mma_commit(&bars[B_D1]);
          // D2 = [T;P] X   (K-dim = tokens: 4 steps)
          ok = wait_shared_bar<kPair>(bars, B_TP_READY + rb, (uint32_t)(n / NTP) & 1u) &&
               wait_bar(bars, B_X_READY, (uint32_t)n & 1u);
          if (!ok) break;
          tc_fence_after();
  #pragma unroll (kPair ? 4 : 1)
          for (int k = 0; k < 4; ++k) {
            const uint64_t a = umma_desc(tp + k * 32, 16, 1024, SW128);
            const uint64_t bd = umma_desc(sbase + SM_X + k * 2048, 8192, 1024, SW128);
            mma_bf16(tmem + TM_D2, a, bd, IDESC_KM, k > 0);
          }
          mma_commit(&bars[B_D2]);
          // D3 = K^T V''  (A MN-major: M = dk in two 64-wide blocks 16 KB apart)
          ok = wait_bar(bars, B_VPP_READY, (uint32_t)n & 1u);
          if (!ok) break;
          tc_fence_after();
          // (DK = 256: rows 128-255 of the increment, key blocks 2-3, into TM_D3 + 128)
  #pragma unroll
          for (int rg = 0; rg < RG; ++rg) {
  #pragma unroll (kPair ? 4 : 1)
            for (int k = 0; k < 4; ++k) {
              const uint64_t a = umma_desc(kq + rg * 32768 + k * 2048, 16384, 1024, SW128);
              const uint64_t bd = umma_desc(sbase + SM_VPP + k * 2048, 8192, 1024, SW128);
              mma_bf16(tmem + TM_D3 + (uint32_t)rg * 128, a, bd, IDESC_MM, k > 0);
            }
          }
          mma_commit(&bars[B_D3]);
          mma_commit(&bars[B_EMPTY + s]);  // K, Q, V of this stage are no longer read
          // D4 = [T;P] V'
          if (n > 0) ok = wait_bar(bars, B_D4_EMPTY, (uint32_t)(n - 1) & 1u);
          if (!ok) break;
          tc_fence_after();
  #pragma unroll (kPair ? 4 : 1)
          for (int k = 0; k < 4; ++k) {
            const uint64_t a = umma_desc(tp + k * 32, 16, 1024, SW128);
            const uint64_t bd = umma_desc(sbase + SM_VP + k * 2048, 8192, 1024, SW128);
            mma_bf16(tmem + TM_D4, a, bd, IDESC_KM, k > 0);
          }
          mma_commit(&bars[B_D4]);
        }
        mma_commit(&bars[B_CHAIN_DONE]);
        wait_bar(bars, B_CHAIN_DONE, 0);
      }
    } else if (warp == 2) {
      // ------------------------------ prep MMA issuer ------------------------------
      if (elect_one()) {
        bool ok = true;
        for (int n = rank, j = 0; n < N && ok; n += step, ++j) {
          const int s = n % NSTAGE, pb = j & 1;
          ok = wait_bar(bars, B_FULL + s, (uint32_t)(n / NSTAGE) & 1u);
          if (ok && j >= 2) ok = wait_bar(bars, B_PRE_EMPTY + pb, (uint32_t)((j - 2) >> 1) & 1u);
          if (!ok) break;
          tc_fence_after();
          const uint32_t kq = sbase + SM_KQ + s * KQ_STAGE;
  #pragma unroll (kPair ? 8 : 1)
          for (int k = 0; k < KSTEPS; ++k) {
            const uint64_t a = umma_desc(kq + (k >> 2) * 16384 + (k & 3) * 32, 16, 1024, SW128);
            mma_bf16(tmem + TM_PRE + (uint32_t)pb * 64, a, a, IDESC_KK, k > 0);
          }
          mma_commit(&bars[B_PRE_FULL + pb]);
        }
      }
    } else if (warp == 3) {
      // ------------------------------ gate warp ------------------------------
      // Per chunk, as soon as its buffer is free (NTP - 1 chunks ahead of the chain):
      // g and beta, then the gate vectors of chunk_gate_vectors.
      const size_t gb = ((size_t)b * T + tok0) * H + h;
      // layer form: g = -exp(A_log[h]) softplus(a + dt_bias[h]), beta = sigmoid(b)
      const float negA = kGates ? -expf(ldg_f32(la.A_log + h)) : 0.f;
      const float dtb = kGates ? ldg_f32(la.dt_bias + h) : 0.f;
      auto gate_of = [&](float x) { return kGates ? negA * softplus(x + dtb) : x; };
      auto beta_of = [&](float x) { return kGates ? sigmoid(x) : x; };
      bool ok = true;
      for (int n = 0; n < N && ok; ++n) {
        const int rb = n % NTP;
        VecBuf& vb = vecs[rb];
        const int t = n * C + 2 * lane;
        const float g0 = t < Tn ? gate_of(ldg_f32(g + gb + (size_t)t * H)) : 0.f;
        const float g1 = t + 1 < Tn ? gate_of(ldg_f32(g + gb + (size_t)(t + 1) * H)) : 0.f;
        const float b0 = t < Tn ? beta_of(ldg_f32(beta + gb + (size_t)t * H)) : 0.f;
        const float b1 = t + 1 < Tn ? beta_of(ldg_f32(beta + gb + (size_t)(t + 1) * H)) : 0.f;
        if (n >= NTP) ok = wait_bar(bars, B_VEC_EMPTY + rb, (uint32_t)((n / NTP) - 1) & 1u);
        if (!ok) break;
        // (the gate factors only serve chunks this CTA prepares)
        chunk_gate_vectors(vb, g0, g1, b0, b1, (n - rank) % step == 0, lane);
        if (lane == 0) mbar_arrive(&bars[B_VEC_FULL + rb]);
      }
    }
  } else if (warp < 12) {
    // ------------------------------ prep (eight warps) ------------------------------
    const int pi = tid - 128;           // 0..255
    const int wq = warp & 3;            // TMEM lane quarter
    const int ch = (warp - 4) >> 2;     // which 32 of the 64 D_pre columns
    const int p = wq * 32 + lane;       // TMEM lane = row of D_pre
    // The strictly upper 16x16 blocks of T are never written below: zero them once.
    for (int e = pi; e < NTP * 64 * 8; e += 256) {
      const int buf = e / 512, row = (e / 8) % 64, c8 = e % 8;
      if (c8 >= 2 * (row / 16 + 1))
        *reinterpret_cast<uint4*>(sm + SM_TP + buf * 16384 + sw128(row, c8)) =
            make_uint4(0u, 0u, 0u, 0u);
    }
    float* AF = reinterpret_cast<float*>(sm + SM_AF);
    float* TF = reinterpret_cast<float*>(sm + SM_TF);
    bool ok = true;
    int last = -1;  // last chunk whose tile was published
    for (int n = rank, oc = 0; n < N && ok; n += step, ++oc) {
      const int pb = oc & 1, rb = n % NTP;  // D_pre buffer, ring slot
      VecBuf& vb = vecs[rb];
      unsigned char* tpt = sm + SM_TP + rb * 16384;
      // ring slot free in every chain of the pair (chunk n - NTP released)
      if (n >= NTP)
        ok = wait_shared_bar<kPair>(bars, B_TP_EMPTY + rb, (uint32_t)((n / NTP) - 1) & 1u);
      if (!ok) break;
      ok = wait_bar(bars, B_VEC_FULL + rb, (uint32_t)(n / NTP) & 1u);
      if (!ok) break;
      const bool direct = vb.direct != 0;
      // A (rows 0-63) and P (rows 64-127) from D_pre; this warp: 32 columns, in
      // steps of kW columns.  Steep gates (direct) form each e^{G_i - G_j}
      // from its own exponent instead of the separable factors.
      const int i = p & 63;
      const int jmax = p < 64 ? i - 1 : i;  // A is strictly lower, P includes the diagonal
      const float rs = p < 64 ? vb.beta[i] : 1.f;
      const float Gi = vb.G[i];
      // (paired form: the factors of the whole 32-column half are formed while
      // the product may still be in flight)
      float fac[kPair ? 32 : 1];
      if constexpr (kPair) {
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          const float fq = rs * vb.F[i][2 * ch + h2];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int j = (2 * ch + h2) * 16 + e;
            fac[16 * h2 + e] =
                (j <= jmax) ? (direct ? rs * gate_exp(Gi - vb.G[j]) : fq * vb.E[j]) : 0.f;
          }
        }
      }
      ok = wait_bar(bars, B_PRE_FULL + pb, (uint32_t)(oc >> 1) & 1u);
      if (!ok) break;
      tc_fence_after();
      {
        const uint32_t ta =
            tmem + TM_PRE + (uint32_t)pb * 64 + (uint32_t)ch * 32 + ((uint32_t)(wq * 32) << 16);
#pragma unroll 1
        for (int cw = 0; cw < 32; cw += kWP) {
          float vrow[kWP];
          tmem_ldw<kWP>(ta + cw, vrow);
#pragma unroll
          for (int h2 = 0; h2 < kWP / 16; ++h2) {
            const int q4 = 2 * ch + cw / 16 + h2;
            const float* v = vrow + 16 * h2;
            float out[16];
            if constexpr (kPair) {
#pragma unroll
              for (int e = 0; e < 16; ++e) out[e] = fac[16 * h2 + e] * v[e];
            } else if (direct) {
#pragma unroll
              for (int e = 0; e < 16; ++e) {
                const int j = q4 * 16 + e;
                out[e] = (j <= jmax) ? rs * gate_exp(Gi - vb.G[j]) * v[e] : 0.f;
              }
            } else {
              const float fq = rs * vb.F[i][q4];
#pragma unroll
              for (int e = 0; e < 16; ++e) {
                const int j = q4 * 16 + e;
                out[e] = (j <= jmax) ? fq * vb.E[j] * v[e] : 0.f;
              }
            }
            if (p < 64) {
#pragma unroll
              for (int e = 0; e < 16; e += 4)
                *reinterpret_cast<float4*>(AF + i * LDF + q4 * 16 + e) =
                    make_float4(rtf32(out[e]), rtf32(out[e + 1]), rtf32(out[e + 2]),
                                rtf32(out[e + 3]));
            } else {
              *reinterpret_cast<uint4*>(tpt + sw128(p, 2 * q4)) = pack_bf16x8(out);
              *reinterpret_cast<uint4*>(tpt + sw128(p, 2 * q4 + 1)) = pack_bf16x8(out + 8);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[B_PRE_EMPTY + pb]);
      named_sync(1, 256);
      // ---- T = (I + A)^{-1}: 16x16 diagonal blocks by column-oriented substitution ----
      if (pi < 64) solve_diag(AF, TF, tpt, nullptr, vb.dec, pi);
      named_sync(1, 256);
      // ---- off-diagonal 16x16 blocks in three phases of independent warp tasks
      //      (tf32 warp MMAs); the schedule is kSolveTask ----
      solve_offdiag(AF, TF, tpt, nullptr, vb.dec, warp - 4, lane, 1, 256);
      // publish the tile: here, and (pair) by a bulk copy into the other CTA's
      // ring slot, completing on its barrier
      fence_proxy_async_smem();
      named_sync(1, 256);
      if (pi == 0) {
        mbar_arrive(&bars[B_TP_READY + rb]);
        if (kPair) {
          const uint32_t tp_local = sbase + SM_TP + rb * 16384;
          const uint32_t bar_peer = mapa_shared(smem_u32(&bars[B_TP_READY + rb]), peer);
          mbar_arrive_expect_tx_cluster_relaxed(bar_peer, 16384);
          bulk_s2s_cluster(mapa_shared(tp_local, peer), tp_local, 16384, bar_peer);
        }
      }
      last = n;
    }
    if (kPair && pi == 0) {
      // Before the CTA can exit, the tiles it copied out into ring slots that no
      // later chunk reuses have been released by both chains, so no copy is
      // still in flight (bounded waits; earlier copies were released before
      // their slot was refilled).
      for (int n = rank; n <= last; n += step)
        if (n + NTP >= N)
          wait_shared_bar<kPair>(bars, B_TP_EMPTY + n % NTP, (uint32_t)(n / NTP) & 1u);
    }
  } else {
    // ------------------------------ chain warpgroup ------------------------------
    regs_increase<kRegsChain>();
    const int r = tid - 384;          // TMEM lane / row
    const int wq = warp - 12;
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    unsigned char* Stile = sm + SM_S;
    // state rows r (and, DK = 256, r + 128) of this column tile
    float S[RG][DVT];
#pragma unroll
    for (int rg = 0; rg < RG; ++rg) {
      const int row = r + 128 * rg;
      const float* src = h0 ? h0 + ((size_t)bh * DK + row) * dv + c0 : nullptr;
#pragma unroll
      for (int c = 0; c < DVT; c += 4) {
        const float4 v = src ? *reinterpret_cast<const float4*>(src + c)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
        S[rg][c] = v.x; S[rg][c + 1] = v.y; S[rg][c + 2] = v.z; S[rg][c + 3] = v.w;
      }
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8)
        *reinterpret_cast<uint4*>(Stile + sw128(row, c8)) = pack_bf16x8(S[rg] + c8 * 8);
    }
    {
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[B_S_READY]);
    }
    // layer form: the norm weight of this column tile, for the output warps
    const bool gated = kLayer && la.gate != nullptr;
    if constexpr (kLayer) {
      if (wq >= 2) {
        reinterpret_cast<float*>(sm + SM_W)[r - 64] = ldg_f32(la.weight + c0 + r - 64);
        named_sync(2, 64);
      }
    }
    // Layer form, output warps: the row of chunk m is finished at the start of
    // chunk m + 1 (or after the last chunk), where these warps would otherwise
    // wait for D3: by then the other CTA's partial sum has long arrived.  Its
    // 64 gate values are fetched at the start of chunk m, a whole chain step
    // before they are used; the bf16 row waits in SM_OB (128-byte swizzled
    // rows, each thread its own row).
    uint4 zr[8];
    float ss_own = 0.f;
    auto fetch_gate = [&](int m) {
      const int t = m * C + r - 64;
      const bool have = gated && t < Tn;
      const uint4* zp =
          have ? reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(la.gate) +
                                                (((size_t)b * T + tok0 + t) * H + h) * dv + c0)
               : nullptr;
#pragma unroll
      for (int j = 0; j < 8; ++j) zr[j] = have ? ldg_u4(zp + j) : make_uint4(0u, 0u, 0u, 0u);
    };
    auto finish_row = [&](int m) -> bool {
      const int i = r - 64, t = m * C + i, sb = m % NSS;
      if (!mbar_wait_cluster(&bars[B_SS + sb], (uint32_t)(m / NSS) & 1u)) return false;
      const float* ssb = reinterpret_cast<const float*>(sm + SM_SS) + sb * 64;
      const float rs = rsqrtf((ss_own + ssb[i]) * (1.f / (2 * DVT)) + la.eps);
      const float* wsm = reinterpret_cast<const float*>(sm + SM_W);
      __nv_bfloat16* orow = o + (((size_t)b * T + tok0 + t) * H + h) * dv + c0;
      // (rolled: this runs in slack time, and instruction fetch is what a CTA
      // pair's SMs compete for)
#pragma unroll 1
      for (int q8 = 0; q8 < 8; ++q8) {
        float x[8], zz[8];
        unpack_bf16x8(*reinterpret_cast<const uint4*>(sm + SM_OB + sw128(i, q8)), x);
        uint4 zq = zr[0];  // zr[q8] by selects, so that zr stays in registers
#pragma unroll
        for (int j = 1; j < 8; ++j) zq = q8 == j ? zr[j] : zq;
        unpack_bf16x8(zq, zz);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float gf = gated ? silu_fast(zz[e]) : 1.f;
          x[e] *= rs * wsm[q8 * 8 + e] * gf;
        }
        if (t < Tn) *reinterpret_cast<uint4*>(orow + q8 * 8) = pack_bf16x8(x);
      }
      return true;
    };
    bool ok = true;
    for (int n = 0; n < N && ok; ++n) {
      const int s = n % NSTAGE, tb = n & 1, rb = n % NTP;
      const VecBuf& vb = vecs[rb];
      const int t0 = n * C;
      const uint32_t d1 = tmem + TM_D1 + (uint32_t)tb * 64 + lane_off;
      if constexpr (kLayer) {
        if (wq >= 2) {
          if (n > 0 && !finish_row(n - 1)) {
            ok = false;
            break;
          }
          fetch_gate(n);
        }
      }
      if (wq < 2) {
        // ---- epilogue 1: X = beta (V - e^G K S) ----
        const int i = r;
        ok = wait_bar(bars, B_D1, (uint32_t)n & 1u) &&
             wait_bar(bars, B_FULL + s, (uint32_t)(n / NSTAGE) & 1u) &&
             wait_bar(bars, B_VEC_FULL + rb, (uint32_t)(n / NTP) & 1u);
        if (!ok) break;
        tc_fence_after();
        const float bi = vb.beta[i], egi = vb.eG[i];
        const unsigned char* Vt = sm + SM_V + s * 8192;
#pragma unroll 1
        for (int cw = 0; cw < DVT; cw += kWC) {
          float ksrow[kWC];
          tmem_ldw<kWC>(d1 + cw, ksrow);
#pragma unroll
          for (int qq = 0; qq < kWC / 16; ++qq) {
            const int q4 = cw / 16 + qq;
            float vv[16], x[16];
            const float* ks = ksrow + 16 * qq;
            unpack_bf16x8(*reinterpret_cast<const uint4*>(Vt + sw128(i, 2 * q4)), vv);
            unpack_bf16x8(*reinterpret_cast<const uint4*>(Vt + sw128(i, 2 * q4 + 1)), vv + 8);
#pragma unroll
            for (int e = 0; e < 16; ++e) x[e] = bi * (vv[e] - egi * ks[e]);
            *reinterpret_cast<uint4*>(sm + SM_X + sw128(i, 2 * q4)) = pack_bf16x8(x);
            *reinterpret_cast<uint4*>(sm + SM_X + sw128(i, 2 * q4 + 1)) = pack_bf16x8(x + 8);
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[B_X_READY]);
        // ---- epilogue 2: V' and V'' = e^{G_C - G} V' ----
        ok = wait_bar(bars, B_D2, (uint32_t)n & 1u);
        if (!ok) break;
        tc_fence_after();
        const float di = vb.dec[i];
#pragma unroll 1
        for (int cw = 0; cw < DVT; cw += kWC) {
          float vprow[kWC];
          tmem_ldw<kWC>(tmem + TM_D2 + lane_off + cw, vprow);
#pragma unroll
          for (int qq = 0; qq < kWC / 16; ++qq) {
            const int q4 = cw / 16 + qq;
            float vpp[16];
            const float* vp = vprow + 16 * qq;
#pragma unroll
            for (int e = 0; e < 16; ++e) vpp[e] = di * vp[e];
            *reinterpret_cast<uint4*>(sm + SM_VPP + sw128(i, 2 * q4)) = pack_bf16x8(vpp);
            *reinterpret_cast<uint4*>(sm + SM_VPP + sw128(i, 2 * q4 + 1)) = pack_bf16x8(vpp + 8);
            *reinterpret_cast<uint4*>(sm + SM_VP + sw128(i, 2 * q4)) = pack_bf16x8(vp);
            *reinterpret_cast<uint4*>(sm + SM_VP + sw128(i, 2 * q4 + 1)) = pack_bf16x8(vp + 8);
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[B_VPP_READY]);
      }
      // ---- epilogue 3: S <- e^{G_C} S + K^T V''  (all DK rows) ----
      // (warps 2-3 read the gate vectors from here on: acquire them directly)
      ok = wait_bar(bars, B_D3, (uint32_t)n & 1u) &&
           (wq < 2 || wait_bar(bars, B_VEC_FULL + rb, (uint32_t)(n / NTP) & 1u));
      if (!ok) break;
      tc_fence_after();
      if constexpr (DK == 128) {
        const float egc = vb.eGC;
        float dsrow[64];
        tmem_ld64(tmem + TM_D3 + lane_off, dsrow);
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const float* ds = dsrow + 16 * q4;
          float* Sr = S[0];
#pragma unroll
          for (int e = 0; e < 16; ++e) Sr[q4 * 16 + e] = fmaf(egc, Sr[q4 * 16 + e], ds[e]);
          *reinterpret_cast<uint4*>(Stile + sw128(r, 2 * q4)) = pack_bf16x8(Sr + q4 * 16);
          *reinterpret_cast<uint4*>(Stile + sw128(r, 2 * q4 + 1)) = pack_bf16x8(Sr + q4 * 16 + 8);
        }
      } else {
        // (two row groups: 32 columns of the increment per TMEM read, to stay
        // within the chain's registers next to the 128 state values)
        const float egc = vb.eGC;
#pragma unroll
        for (int rg = 0; rg < RG; ++rg) {
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            float ds[32];
            tmem_ld32(tmem + TM_D3 + (uint32_t)rg * 128 + lane_off + h2 * 32, ds);
            float* Sr = S[rg] + 32 * h2;
#pragma unroll
            for (int e = 0; e < 32; ++e) Sr[e] = fmaf(egc, Sr[e], ds[e]);
#pragma unroll
            for (int c8 = 0; c8 < 4; ++c8)
              *reinterpret_cast<uint4*>(Stile + sw128(r + 128 * rg, 4 * h2 + c8)) =
                  pack_bf16x8(Sr + 8 * c8);
          }
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[B_S_READY]);
      if (wq >= 2) {
        // ---- epilogue 4: O = e^G (Q S) + P V'  (rows 64-127 of D1 and D4) ----
        const int i = r - 64;
        ok = wait_bar(bars, B_D4, (uint32_t)n & 1u);
        if (!ok) break;
        tc_fence_after();
        const float egi = vb.eG[i];
        const int t = t0 + i;
        __nv_bfloat16* orow = o + (((size_t)b * T + tok0 + t) * H + h) * dv + c0;
        if constexpr (kLayer) {
          // ---- layer form, first half: y = O rsqrt(mean(O^2) + eps) w silu(gate)
          //      over the row's 128 columns, 64 here and 64 in the other CTA of the
          //      pair.  One pass over TMEM sums the squares of the fp32 row and
          //      stages it as bf16 (as the op's own output would be); the partial
          //      sum goes to the other CTA, and TMEM is released at once. ----
          float ss = 0.f;
#pragma unroll 1
          for (int q4 = 0; q4 < 4; ++q4) {
            float qs[16], pv[16];
            tmem_ld16x2(d1 + q4 * 16, tmem + TM_D4 + lane_off + q4 * 16, qs, pv);
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              qs[e] = fmaf(egi, qs[e], pv[e]);
              ss = fmaf(qs[e], qs[e], ss);
            }
            *reinterpret_cast<uint4*>(sm + SM_OB + sw128(i, 2 * q4)) = pack_bf16x8(qs);
            *reinterpret_cast<uint4*>(sm + SM_OB + sw128(i, 2 * q4 + 1)) = pack_bf16x8(qs + 8);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars[B_D4_EMPTY]);
          const int sb = n % NSS;
          st_async_cluster_f32(
              mapa_shared(smem_u32(reinterpret_cast<float*>(sm + SM_SS) + sb * 64 + i), peer), ss,
              mapa_shared(smem_u32(&bars[B_SS + sb]), peer));
          if (i == 0) mbar_arrive_expect_tx(&bars[B_SS + sb], 64 * 4);
          ss_own = ss;
        } else {
#pragma unroll (kPair ? 4 : 1)
          for (int q4 = 0; q4 < 4; ++q4) {
            float qs[16], pv[16], out[16];
            tmem_ld16(d1 + q4 * 16, qs);
            tmem_ld16(tmem + TM_D4 + lane_off + q4 * 16, pv);
#pragma unroll
            for (int e = 0; e < 16; ++e) out[e] = fmaf(egi, qs[e], pv[e]);
            if (t < Tn) {
              *reinterpret_cast<uint4*>(orow + q4 * 16) = pack_bf16x8(out);
              *reinterpret_cast<uint4*>(orow + q4 * 16 + 8) = pack_bf16x8(out + 8);
            }
          }
        }
        if constexpr (!kLayer) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars[B_D4_EMPTY]);
        }
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bars[B_VEC_EMPTY + rb]);
        mbar_arrive(&bars[B_TP_EMPTY + rb]);
        // (the tile's last reader, D4, completed before this warp went on)
        if (kPair)
          mbar_arrive_cluster_relaxed(mapa_shared(smem_u32(&bars[B_TP_EMPTY + rb]), peer));
      }
    }
    if constexpr (kLayer) {
      if (ok && wq >= 2 && N > 0) ok = finish_row(N - 1);
    }
    if (ok && hT) {
#pragma unroll
      for (int rg = 0; rg < RG; ++rg) {
        float* dst = hT + ((size_t)bh * DK + r + 128 * rg) * dv + c0;
#pragma unroll
        for (int c = 0; c < DVT; c += 4)
          *reinterpret_cast<float4*>(dst + c) =
              make_float4(S[rg][c], S[rg][c + 1], S[rg][c + 2], S[rg][c + 3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  // neither CTA of a cluster leaves while the other may still reach its shared memory
  if (kCluster) cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TM_COLS);
  }
}

}  // namespace

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// [B, T, H, D] bf16 viewed as a 4-D tensor (D, H, T, B); box = 64 x 1 x 64 x 1.
bool make_bf16_map_4d(CUtensorMap* m, const void* base, int B, int T, int H, int D) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)D * 2, (cuuint64_t)H * D * 2, (cuuint64_t)T * H * D * 2};
  cuuint32_t box[4] = {64, 1, 64, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// [rows, D] fp32 row-major as a 2-D TMA map (D, rows), boxes of 32 x 32 with
// 128-byte swizzle (a box row is 128 bytes).
bool make_f32_map_2d(CUtensorMap* m, const void* base, long long rows, int D) {
  auto fn = encode_fn();
  if (!fn || rows <= 0 || D % 32 != 0) return false;
  cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)D * 4};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// [rows, D] bf16 row-major as a 2-D TMA map (D, rows) with boxes of bx x by:
// 64 x 64 with 128-byte swizzle (swizzled = true; tile loads), or 32 x 32
// unswizzled (64-byte box rows; tile stores from row-major staging).
bool make_bf16_map_2d(CUtensorMap* m, const void* base, long long rows, int D, bool swizzled) {
  auto fn = encode_fn();
  if (!fn || rows <= 0 || D % 64 != 0) return false;
  cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)D * 2};
  cuuint32_t box[2] = {swizzled ? 64u : 32u, swizzled ? 64u : 32u};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzled ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

GDN_DEVICE_ERROR_ACCESSOR(device_error_chunk_tc)

// Exact semantics compute the recurrence whatever the chunk length, so this
// kernel (chunks of 64) serves every requested chunk size; only the
// reference-literal semantics depend on the chunk length (partial-chunk decay,
// output order) and stay with the CUDA-core kernel.
bool chunk_tc_supported(const ChunkArgs& a) {
  return a.dtype == kBF16 && a.semantics == kExact && (a.dk == 128 || a.dk == 256) &&
         a.dv % DVT == 0 && a.T > 0 && encode_fn() != nullptr;
}

namespace {

template <int DK, bool kPair, bool kLayer, bool kGates = kLayer>
cudaError_t launch_tc_form(const ChunkArgs& a, const LayerArgs& la, cudaStream_t st) {
  constexpr int SMEM_BYTES = Lay<DK>::SMEM_BYTES;
  CUtensorMap mk, mq, mv;
  const int rows = a.cu_seqlens ? 1 : a.B;  // packed sequences share one row of T tokens
  if (!make_bf16_map_4d(&mk, a.k, rows, a.T, a.Hk, a.dk) ||
      !make_bf16_map_4d(&mq, a.q, rows, a.T, a.Hk, a.dk) ||
      !make_bf16_map_4d(&mv, a.v, rows, a.T, a.H, a.dv))
    return cudaErrorInvalidValue;
  auto kernel = chunk_tc_kernel<DK, kPair, kLayer, kGates>;
  // The in-kernel register split assumes exactly kLaunchRegs per thread at
  // launch; with fewer, the chain warpgroup's increase could never be granted.
  // (Checked, and shared memory opted in, once per device and form.)
  static std::atomic<int> slot[kMaxDevices] = {};
  cudaError_t e = cudaSuccess;
  if (slot[current_device()].load(std::memory_order_acquire) < SMEM_BYTES) {
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, kernel);
    if (e != cudaSuccess) return e;
    if (fa.numRegs != kLaunchRegs) return cudaErrorInvalidConfiguration;
  }
  e = ensure_smem(kernel, SMEM_BYTES, slot);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.dv / DVT, a.B * a.H);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (kPair || kLayer) ? 2 : 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kernel, mk, mq, mv, a.g, a.beta, a.h0,
                         static_cast<__nv_bfloat16*>(a.o), a.hT, a.cu_seqlens, a.T, a.H, a.Hk,
                         a.dv, la);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_chunk_tc(const ChunkArgs& a, cudaStream_t st) {
  if (a.B * a.H == 0 || a.T == 0) return cudaSuccess;
  // Pairs of column tiles share the preparation (clusters of two CTAs) when
  // the tile count is even and the grid leaves every CTA pair a TPC (two SMs)
  // of its own; at higher occupancy the SMs of a TPC compete for instruction
  // fetch and the compact unpaired kernel is faster.  GDN_CHUNK_TC_PAIR=0 / 1
  // forces either form (kernel cross-checks).
  const int tiles = a.dv / DVT;
  const long long ctas = (long long)tiles * a.B * a.H;
  const int sms = device_sm_count();
  const int force = kernel_overrides().tc_pair;
  bool pair = tiles % 2 == 0 && ctas <= sms / 2;
  if (force == 0) pair = false;
  if (force == 1) pair = tiles % 2 == 0;
  const LayerArgs none;
  // (DK = 256: the unpaired form only)
  if (a.dk == 256) return launch_tc_form<256, false, false>(a, none, st);
  return pair ? launch_tc_form<128, true, false>(a, none, st)
              : launch_tc_form<128, false, false>(a, none, st);
}

// The layer form always runs the two 64-column tiles of a row as one cluster:
// the norm of a row needs both halves.  The two CTAs also share the
// preparation at low occupancy; the layer form's larger code makes the compact
// form win from fewer CTAs than the op's rule (measured: pairs at 32 CTAs,
// 216 against 244 us; compact at 64, 238 against 248 us).  GDN_CHUNK_TC_PAIR
// forces either form.
cudaError_t launch_chunk_tc_layer(const ChunkArgs& a, const LayerArgs& la, cudaStream_t st) {
  if (a.B * a.H == 0 || a.T == 0) return cudaSuccess;
  if (!chunk_tc_supported(a) || a.dk != 128 || a.dv != 2 * DVT) return cudaErrorInvalidValue;
  const long long ctas = 2LL * a.B * a.H;
  const int force = kernel_overrides().tc_pair;
  bool pair = ctas <= device_sm_count() / 3;
  if (force == 0) pair = false;
  if (force == 1) pair = true;
  return pair ? launch_tc_form<128, true, true>(a, la, st)
              : launch_tc_form<128, false, true>(a, la, st);
}

// The gates-only form (compact, unpaired): g and beta from the raw
// projections in the gate warp, o as the op writes it.  The layer at the
// other tcgen05 shapes (dk = 256, or dv other than 128) runs this and then a
// gated RMSNorm over o.
cudaError_t launch_chunk_tc_gates(const ChunkArgs& a, const LayerArgs& la, cudaStream_t st) {
  if (a.B * a.H == 0 || a.T == 0) return cudaSuccess;
  if (!chunk_tc_supported(a)) return cudaErrorInvalidValue;
  if (a.dk == 256) return launch_tc_form<256, false, false, true>(a, la, st);
  return launch_tc_form<128, false, false, true>(a, la, st);
}

}  // namespace gdn
