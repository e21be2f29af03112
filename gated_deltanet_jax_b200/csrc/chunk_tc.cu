// Chunked gated delta-rule forward on 5th-generation tensor cores, sm_100a.
//
// Replaces chunk_gated_delta_rule_fwd (ops.py:299-346) for bf16 inputs with
// dk = 128, dv a multiple of 64 and chunk = 64 (exact semantics).  Every
// matrix product is a tcgen05.mma (bf16 operands in shared memory, fp32
// accumulators in tensor memory) fed by TMA tile loads; the state stays on
// chip for the whole sequence.
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
// Warp roles (384 threads): warp 0 issues TMA loads, warp 1 the chain MMAs
// and owns the tensor memory, warp 2 the prep MMAs; warps 4-7 do the prep
// math, warps 8-11 the chain epilogues.  A warp reads only its own quarter of
// the 128 TMEM lanes, so row r of every M=128 accumulator belongs to thread r
// of a warpgroup.  All hand-offs are mbarriers; every wait is bounded.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "gdn_common.cuh"
#include "gdn_internal.h"
#include "ptx.cuh"

namespace gdn {

namespace {

constexpr int C = 64;
constexpr int DK = 128;
constexpr int DVT = 64;
constexpr int NSTAGE = 2;
constexpr int kThreads = 384;
constexpr int LDF = 68;  // fp32 row stride of the A / T matrices (16-byte aligned rows)
constexpr int LDY = 20;  // fp32 row stride of the per-warp 16x16 scratch

// Shared-memory byte offsets from a 1024-byte aligned base.
constexpr int SM_KQ = 0;                        // NSTAGE x [2 kblk][128 rows][128 B]
constexpr int SM_V = SM_KQ + NSTAGE * 32768;    // NSTAGE x [64 rows][128 B]
constexpr int SM_S = SM_V + NSTAGE * 8192;      // [128 rows (dk)][128 B]
constexpr int SM_X = SM_S + 16384;              // [64 rows (token)][128 B]
constexpr int SM_VPP = SM_X + 8192;             // V'' = e^{G_C-G} V'
constexpr int SM_VP = SM_VPP + 8192;            // V'
constexpr int SM_TP = SM_VP + 8192;             // 2 x [128 rows][128 B]: rows 0-63 T, 64-127 P
constexpr int SM_AF = SM_TP + 2 * 16384;        // fp32 A [64][LDF]
constexpr int SM_TF = SM_AF + 64 * LDF * 4;     // fp32 T [64][LDF]
constexpr int SM_Y = SM_TF + 64 * LDF * 4;      // fp32 [3 warps][16][LDY]
constexpr int SM_VEC = SM_Y + 3 * 16 * LDY * 4; // 2 x VecBuf
struct VecBuf {
  float G[C], eG[C], dec[C], beta[C];
  float F[C][4];  // e^{G_i - G_{16k}} for k <= i / 16 (gate factors, row part)
  float E[C];     // e^{G_{16 floor(j/16)} - G_j}      (gate factors, column part)
  float eGC, pad[3];
};
constexpr int SM_BAR = SM_VEC + 2 * (int)sizeof(VecBuf);
constexpr int NBAR = 24;
constexpr int SM_TMEM = SM_BAR + NBAR * 8;
constexpr int SM_TOTAL = SM_TMEM + 16;
constexpr int SMEM_BYTES = SM_TOTAL + 1024;  // + alignment slack
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");

// barrier indices
enum {
  B_FULL = 0,        // [NSTAGE] TMA stage loaded
  B_EMPTY = 2,       // [NSTAGE] stage consumed by the MMAs
  B_PRE_FULL = 4,    // [2] D_pre ready
  B_PRE_EMPTY = 6,   // [2] D_pre read by prep
  B_TP_READY = 8,    // [2] TP tile + vectors of a chunk ready
  B_TP_EMPTY = 10,   // [2] chain done with a chunk's TP / vectors
  B_D1 = 12, B_D2 = 13, B_D3 = 14, B_D4 = 15, B_D4_EMPTY = 16,
  B_X_READY = 17, B_VPP_READY = 18, B_S_READY = 19, B_CHAIN_DONE = 20,
};

// TMEM columns
constexpr uint32_t TM_PRE = 0;    // 2 x 64
constexpr uint32_t TM_D1 = 128;   // 2 x 64
constexpr uint32_t TM_D2 = 256;
constexpr uint32_t TM_D3 = 320;
constexpr uint32_t TM_D4 = 384;
constexpr uint32_t TM_COLS = 512;

constexpr uint32_t IDESC_KK = idesc_bf16(128, 64, 0, 0);  // A K-major, B K-major
constexpr uint32_t IDESC_KM = idesc_bf16(128, 64, 0, 1);  // A K-major, B MN-major
constexpr uint32_t IDESC_MM = idesc_bf16(128, 64, 1, 1);  // A MN-major, B MN-major
constexpr uint32_t SW128 = 2;

__device__ __forceinline__ uint4 pack_bf16x8(const float* f) {
  uint4 u;
  __nv_bfloat162 t0 = __floats2bfloat162_rn(f[0], f[1]);
  __nv_bfloat162 t1 = __floats2bfloat162_rn(f[2], f[3]);
  __nv_bfloat162 t2 = __floats2bfloat162_rn(f[4], f[5]);
  __nv_bfloat162 t3 = __floats2bfloat162_rn(f[6], f[7]);
  u.x = *reinterpret_cast<uint32_t*>(&t0);
  u.y = *reinterpret_cast<uint32_t*>(&t1);
  u.z = *reinterpret_cast<uint32_t*>(&t2);
  u.w = *reinterpret_cast<uint32_t*>(&t3);
  return u;
}

__device__ __forceinline__ void unpack_bf16x8(uint4 u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 t = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
    float2 p = __bfloat1622float2(t);
    f[2 * i] = p.x;
    f[2 * i + 1] = p.y;
  }
}

__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

// D(16x8) += A(16x8, row) * B(8x8, col), tf32 inputs, fp32 accumulate.
__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4],
                                         const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// OR of `pred` over the 128 threads of the prep warpgroup (named barrier 1).
__device__ __forceinline__ int __syncthreads_or_named(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred)
      : "memory");
  return (int)r;
}

__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Bounded wait by a single thread (the elected lane of a one-thread role).
__device__ __forceinline__ bool wait_bar(uint64_t* bars, int idx, uint32_t parity) {
  return mbar_wait(&bars[idx], parity);
}

__global__ void __launch_bounds__(kThreads, 1)
chunk_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmQ,
                const __grid_constant__ CUtensorMap tmV, const float* __restrict__ g,
                const float* __restrict__ beta, const float* __restrict__ h0,
                __nv_bfloat16* __restrict__ o, float* __restrict__ hT, int T, int H, int dv) {
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
  const int b = bh / H, h = bh - b * H;
  const int c0 = blockIdx.x * DVT;
  const int N = (T + C - 1) / C;

  if (tid == 0) {
    mbar_init(&bars[B_FULL + 0], 1);
    mbar_init(&bars[B_FULL + 1], 1);
    mbar_init(&bars[B_EMPTY + 0], 1);
    mbar_init(&bars[B_EMPTY + 1], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[B_PRE_FULL + i], 1);
      mbar_init(&bars[B_PRE_EMPTY + i], 4);
      mbar_init(&bars[B_TP_READY + i], 4);
      mbar_init(&bars[B_TP_EMPTY + i], 4);
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
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sbase = smem_u32(sm);

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (elect_one()) {
      int issued = 0;
      bool ok = true;
      for (int n = 0; n < N && ok; ++n) {
        const int s = n % NSTAGE;
        if (n >= NSTAGE) ok = wait_bar(bars, B_EMPTY + s, (uint32_t)((n / NSTAGE) - 1) & 1u);
        if (!ok) break;
        unsigned char* kq = sm + SM_KQ + s * 32768;
        uint64_t* fb = &bars[B_FULL + s];
        mbar_arrive_expect_tx(fb, 4 * 8192 + 8192);
        const int t0 = n * C;
        tma_load_4d(kq, &tmK, 0, h, t0, b, fb);
        tma_load_4d(kq + 16384, &tmK, 64, h, t0, b, fb);
        tma_load_4d(kq + 8192, &tmQ, 0, h, t0, b, fb);
        tma_load_4d(kq + 16384 + 8192, &tmQ, 64, h, t0, b, fb);
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
        const int s = n % NSTAGE, tb = n & 1;
        const uint32_t kq = sbase + SM_KQ + s * 32768;
        const uint32_t tp = sbase + SM_TP + tb * 16384;
        ok = wait_bar(bars, B_FULL + s, (uint32_t)(n / NSTAGE) & 1u) &&
             wait_bar(bars, B_S_READY, (uint32_t)n & 1u);
        if (!ok) break;
        tc_fence_after();
        // D1 = [K;Q] S   (K-dim = dk: 8 steps of 16)
        const uint32_t d1 = tmem + TM_D1 + (uint32_t)tb * 64;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint64_t a = umma_desc(kq + (k >> 2) * 16384 + (k & 3) * 32, 16, 1024, SW128);
          const uint64_t bd = umma_desc(sbase + SM_S + k * 2048, 16384, 1024, SW128);
          mma_bf16(d1, a, bd, IDESC_KM, k > 0);
        }
        mma_commit(&bars[B_D1]);
        // D2 = [T;P] X   (K-dim = tokens: 4 steps)
        ok = wait_bar(bars, B_TP_READY + tb, (uint32_t)(n >> 1) & 1u) &&
             wait_bar(bars, B_X_READY, (uint32_t)n & 1u);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
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
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t a = umma_desc(kq + k * 2048, 16384, 1024, SW128);
          const uint64_t bd = umma_desc(sbase + SM_VPP + k * 2048, 8192, 1024, SW128);
          mma_bf16(tmem + TM_D3, a, bd, IDESC_MM, k > 0);
        }
        mma_commit(&bars[B_D3]);
        mma_commit(&bars[B_EMPTY + s]);  // K, Q, V of this stage are no longer read
        // D4 = [T;P] V'
        if (n > 0) ok = wait_bar(bars, B_D4_EMPTY, (uint32_t)(n - 1) & 1u);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
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
      for (int n = 0; n < N && ok; ++n) {
        const int s = n % NSTAGE, pb = n & 1;
        ok = wait_bar(bars, B_FULL + s, (uint32_t)(n / NSTAGE) & 1u);
        if (ok && n >= 2) ok = wait_bar(bars, B_PRE_EMPTY + pb, (uint32_t)((n - 2) >> 1) & 1u);
        if (!ok) break;
        tc_fence_after();
        const uint32_t kq = sbase + SM_KQ + s * 32768;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint64_t a = umma_desc(kq + (k >> 2) * 16384 + (k & 3) * 32, 16, 1024, SW128);
          mma_bf16(tmem + TM_PRE + (uint32_t)pb * 64, a, a, IDESC_KK, k > 0);
        }
        mma_commit(&bars[B_PRE_FULL + pb]);
      }
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------ prep warpgroup ------------------------------
    const int p = tid - 128;          // TMEM lane / row
    const int wq = warp - 4;          // lane quarter
    const size_t gb = (size_t)b * T * H + h;
    float gn0 = 0.f, gn1 = 0.f, bn0 = 0.f, bn1 = 0.f;
    auto fetch = [&](int n) {
      if (p < 32) {
        const int t = n * C + 2 * p;
        gn0 = t < T ? ldg_f32(g + gb + (size_t)t * H) : 0.f;
        gn1 = t + 1 < T ? ldg_f32(g + gb + (size_t)(t + 1) * H) : 0.f;
        bn0 = t < T ? ldg_f32(beta + gb + (size_t)t * H) : 0.f;
        bn1 = t + 1 < T ? ldg_f32(beta + gb + (size_t)(t + 1) * H) : 0.f;
      }
    };
    fetch(0);
    float* AF = reinterpret_cast<float*>(sm + SM_AF);
    float* TF = reinterpret_cast<float*>(sm + SM_TF);
    float* Y = reinterpret_cast<float*>(sm + SM_Y);
    bool ok = true;
    for (int n = 0; n < N && ok; ++n) {
      const int pb = n & 1;
      VecBuf& vb = vecs[pb];
      unsigned char* tpt = sm + SM_TP + pb * 16384;
      if (n >= 2) ok = wait_bar(bars, B_TP_EMPTY + pb, (uint32_t)((n - 2) >> 1) & 1u);
      if (!ok) break;
      // per-chunk vectors: cumulative gate and its exponentials (warp 0)
      if (p < 32) {
        const float pair = gn0 + gn1;
        float incl = pair;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const float y = __shfl_up_sync(0xffffffffu, incl, off);
          if (lane >= off) incl += y;
        }
        const float G0 = incl - pair + gn0, G1 = incl;
        const float GC = __shfl_sync(0xffffffffu, incl, 31);
        vb.G[2 * p] = G0;
        vb.G[2 * p + 1] = G1;
        vb.beta[2 * p] = bn0;
        vb.beta[2 * p + 1] = bn1;
        vb.eG[2 * p] = gate_exp(G0);
        vb.eG[2 * p + 1] = gate_exp(G1);
        vb.dec[2 * p] = gate_exp(GC - G0);
        vb.dec[2 * p + 1] = gate_exp(GC - G1);
        if (p == 0) vb.eGC = gate_exp(GC);
        if (n + 1 < N) fetch(n + 1);
      }
      named_sync(1, 128);
      // Separable gate factors: e^{G_i - G_j} = F[i][j/16] * E[j] for j <= i.
      // Every exponent lies in one 16-token block or spans from a block start
      // to a later row; if any exceeds 40 (a factor could then overflow, or
      // hide a non-negligible product behind an underflowed partner) the
      // chunk forms e^{G_i - G_j} directly instead.
      bool direct;
      {
        const int i = p & 63, k0 = (p >> 6) * 2;
        float big = 0.f;
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const int k = k0 + kk;
          const float x = (16 * k <= i) ? vb.G[i] - vb.G[16 * k] : 0.f;
          vb.F[i][k] = gate_exp(x);
          big = fmaxf(big, x);
        }
        if (p < 64) {
          const float x = vb.G[p & ~15] - vb.G[p];
          vb.E[p] = gate_exp(x);
          big = fmaxf(big, x);
        }
        direct = __syncthreads_or_named(big > 40.f) != 0;
      }
      // A (rows 0-63) and P (rows 64-127) from D_pre
      ok = wait_bar(bars, B_PRE_FULL + pb, (uint32_t)(n >> 1) & 1u);
      if (!ok) break;
      tc_fence_after();
      {
        const int i = p & 63;
        const float Gi = vb.G[i], bi = vb.beta[i];
        const uint32_t ta = tmem + TM_PRE + (uint32_t)pb * 64 + ((uint32_t)(wq * 32) << 16);
#pragma unroll
        const int jmax = p < 64 ? i - 1 : i;  // A is strictly lower, P includes the diagonal
        const float rs = p < 64 ? bi : 1.f;
        for (int q4 = 0; q4 < 4; ++q4) {
          float v[16];
          tmem_ld16(ta + q4 * 16, v);
          float out[16];
          const float fq = rs * vb.F[i][q4];
          if (!direct) {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const int j = q4 * 16 + e;
              out[e] = (j <= jmax) ? fq * vb.E[j] * v[e] : 0.f;
            }
          } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const int j = q4 * 16 + e;
              out[e] = (j <= jmax) ? rs * gate_exp(Gi - vb.G[j]) * v[e] : 0.f;
            }
          }
          if (p < 64) {
#pragma unroll
            for (int e = 0; e < 16; e += 4)
              *reinterpret_cast<float4*>(AF + i * LDF + q4 * 16 + e) =
                  make_float4(out[e], out[e + 1], out[e + 2], out[e + 3]);
          } else {
            *reinterpret_cast<uint4*>(tpt + sw128(p, 2 * q4)) = pack_bf16x8(out);
            *reinterpret_cast<uint4*>(tpt + sw128(p, 2 * q4 + 1)) = pack_bf16x8(out + 8);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[B_PRE_EMPTY + pb]);
      named_sync(1, 128);
      // ---- T = (I + A)^{-1}: 16x16 diagonal blocks by substitution ----
      if (p < 64) {
        const int blk = p >> 4, c = p & 15;
        const float* Ab = AF + (blk * 16) * LDF + blk * 16;
        float t[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
          float acc = 0.f;
#pragma unroll
          for (int j = 0; j < r; ++j) acc = fmaf(Ab[r * LDF + j], t[j], acc);
          t[r] = (r < c) ? 0.f : ((r == c) ? 1.f : -acc);
        }
        float* Tb = TF + (blk * 16) * LDF + blk * 16;
#pragma unroll
        for (int r = 0; r < 16; ++r) Tb[r * LDF + c] = t[r];
      }
      named_sync(1, 128);
      // ---- off-diagonal blocks, one block diagonal at a time:
      //      T_ij = -T_ii sum_{k=j}^{i-1} A_ik T_kj  (warp w: block j = w),
      //      16x16 products on warp-level tf32 MMAs (m16n8k8), fp32 accumulate ----
      {
        const int gq = lane >> 2, tq = lane & 3;
        float* Yw = Y + wq * 16 * LDY;
        for (int L = 1; L < 4; ++L) {
          if (wq < 4 - L) {
            const int jb = wq, ib = jb + L;
            float acc[2][4] = {};
            for (int kb = jb; kb < ib; ++kb) {
#pragma unroll
              for (int kk = 0; kk < 16; kk += 8) {
                const float* Ar = AF + (ib * 16) * LDF + kb * 16 + kk;
                const uint32_t a[4] = {to_tf32(Ar[gq * LDF + tq]), to_tf32(Ar[(gq + 8) * LDF + tq]),
                                       to_tf32(Ar[gq * LDF + tq + 4]),
                                       to_tf32(Ar[(gq + 8) * LDF + tq + 4])};
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) {
                  const float* Tr = TF + (kb * 16 + kk) * LDF + jb * 16 + nt * 8;
                  const uint32_t bb[2] = {to_tf32(Tr[tq * LDF + gq]), to_tf32(Tr[(tq + 4) * LDF + gq])};
                  mma_tf32(acc[nt], a, bb);
                }
              }
            }
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
              Yw[gq * LDY + nt * 8 + 2 * tq] = acc[nt][0];
              Yw[gq * LDY + nt * 8 + 2 * tq + 1] = acc[nt][1];
              Yw[(gq + 8) * LDY + nt * 8 + 2 * tq] = acc[nt][2];
              Yw[(gq + 8) * LDY + nt * 8 + 2 * tq + 1] = acc[nt][3];
            }
            __syncwarp();
            float acc2[2][4] = {};
#pragma unroll
            for (int kk = 0; kk < 16; kk += 8) {
              const float* Tr = TF + (ib * 16) * LDF + ib * 16 + kk;
              const uint32_t a[4] = {to_tf32(Tr[gq * LDF + tq]), to_tf32(Tr[(gq + 8) * LDF + tq]),
                                     to_tf32(Tr[gq * LDF + tq + 4]),
                                     to_tf32(Tr[(gq + 8) * LDF + tq + 4])};
#pragma unroll
              for (int nt = 0; nt < 2; ++nt) {
                const uint32_t bb[2] = {to_tf32(Yw[(kk + tq) * LDY + nt * 8 + gq]),
                                        to_tf32(Yw[(kk + tq + 4) * LDY + nt * 8 + gq])};
                mma_tf32(acc2[nt], a, bb);
              }
            }
            float* Td = TF + (ib * 16) * LDF + jb * 16;
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
              Td[gq * LDF + nt * 8 + 2 * tq] = -acc2[nt][0];
              Td[gq * LDF + nt * 8 + 2 * tq + 1] = -acc2[nt][1];
              Td[(gq + 8) * LDF + nt * 8 + 2 * tq] = -acc2[nt][2];
              Td[(gq + 8) * LDF + nt * 8 + 2 * tq + 1] = -acc2[nt][3];
            }
            __syncwarp();
          }
          named_sync(1, 128);
        }
      }
      // ---- T -> bf16 rows 0-63 of the TP tile (zero above the diagonal) ----
      if (p < 64) {
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          float f[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int j = c8 * 8 + e;
            f[e] = (j <= p) ? TF[p * LDF + j] : 0.f;
          }
          *reinterpret_cast<uint4*>(tpt + sw128(p, c8)) = pack_bf16x8(f);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[B_TP_READY + pb]);
    }
  } else if (warp >= 8) {
    // ------------------------------ chain warpgroup ------------------------------
    const int r = tid - 256;          // TMEM lane / row
    const int wq = warp - 8;
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    unsigned char* Stile = sm + SM_S;
    float S[DVT];
    {
      const float* src = h0 ? h0 + ((size_t)bh * DK + r) * dv + c0 : nullptr;
#pragma unroll
      for (int c = 0; c < DVT; c += 4) {
        const float4 v = src ? *reinterpret_cast<const float4*>(src + c)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
        S[c] = v.x; S[c + 1] = v.y; S[c + 2] = v.z; S[c + 3] = v.w;
      }
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8)
        *reinterpret_cast<uint4*>(Stile + sw128(r, c8)) = pack_bf16x8(S + c8 * 8);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[B_S_READY]);
    }
    bool ok = true;
    for (int n = 0; n < N && ok; ++n) {
      const int s = n % NSTAGE, tb = n & 1;
      const VecBuf& vb = vecs[tb];
      const int t0 = n * C;
      const uint32_t d1 = tmem + TM_D1 + (uint32_t)tb * 64 + lane_off;
      if (wq < 2) {
        // ---- epilogue 1: X = beta (V - e^G K S) ----
        const int i = r;
        ok = wait_bar(bars, B_D1, (uint32_t)n & 1u) &&
             wait_bar(bars, B_TP_READY + tb, (uint32_t)(n >> 1) & 1u) &&
             wait_bar(bars, B_FULL + s, (uint32_t)(n / NSTAGE) & 1u);
        if (!ok) break;
        tc_fence_after();
        const float bi = vb.beta[i], egi = vb.eG[i];
        const unsigned char* Vt = sm + SM_V + s * 8192;
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          float ks[16], vv[16], x[16];
          tmem_ld16(d1 + q4 * 16, ks);
          unpack_bf16x8(*reinterpret_cast<const uint4*>(Vt + sw128(i, 2 * q4)), vv);
          unpack_bf16x8(*reinterpret_cast<const uint4*>(Vt + sw128(i, 2 * q4 + 1)), vv + 8);
#pragma unroll
          for (int e = 0; e < 16; ++e) x[e] = bi * (vv[e] - egi * ks[e]);
          *reinterpret_cast<uint4*>(sm + SM_X + sw128(i, 2 * q4)) = pack_bf16x8(x);
          *reinterpret_cast<uint4*>(sm + SM_X + sw128(i, 2 * q4 + 1)) = pack_bf16x8(x + 8);
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
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          float vp[16], vpp[16];
          tmem_ld16(tmem + TM_D2 + lane_off + q4 * 16, vp);
#pragma unroll
          for (int e = 0; e < 16; ++e) vpp[e] = di * vp[e];
          *reinterpret_cast<uint4*>(sm + SM_VPP + sw128(i, 2 * q4)) = pack_bf16x8(vpp);
          *reinterpret_cast<uint4*>(sm + SM_VPP + sw128(i, 2 * q4 + 1)) = pack_bf16x8(vpp + 8);
          *reinterpret_cast<uint4*>(sm + SM_VP + sw128(i, 2 * q4)) = pack_bf16x8(vp);
          *reinterpret_cast<uint4*>(sm + SM_VP + sw128(i, 2 * q4 + 1)) = pack_bf16x8(vp + 8);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[B_VPP_READY]);
      }
      // ---- epilogue 3: S <- e^{G_C} S + K^T V''  (all 128 rows) ----
      ok = wait_bar(bars, B_D3, (uint32_t)n & 1u);
      if (!ok) break;
      tc_fence_after();
      {
        const float egc = vb.eGC;
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          float ds[16];
          tmem_ld16(tmem + TM_D3 + lane_off + q4 * 16, ds);
#pragma unroll
          for (int e = 0; e < 16; ++e) S[q4 * 16 + e] = fmaf(egc, S[q4 * 16 + e], ds[e]);
          *reinterpret_cast<uint4*>(Stile + sw128(r, 2 * q4)) = pack_bf16x8(S + q4 * 16);
          *reinterpret_cast<uint4*>(Stile + sw128(r, 2 * q4 + 1)) = pack_bf16x8(S + q4 * 16 + 8);
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
        __nv_bfloat16* orow = o + (((size_t)b * T + t) * H + h) * dv + c0;
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          float qs[16], pv[16], out[16];
          tmem_ld16(d1 + q4 * 16, qs);
          tmem_ld16(tmem + TM_D4 + lane_off + q4 * 16, pv);
#pragma unroll
          for (int e = 0; e < 16; ++e) out[e] = fmaf(egi, qs[e], pv[e]);
          if (t < T) {
            *reinterpret_cast<uint4*>(orow + q4 * 16) = pack_bf16x8(out);
            *reinterpret_cast<uint4*>(orow + q4 * 16 + 8) = pack_bf16x8(out + 8);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[B_D4_EMPTY]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[B_TP_EMPTY + tb]);
    }
    if (ok && hT) {
      float* dst = hT + ((size_t)bh * DK + r) * dv + c0;
#pragma unroll
      for (int c = 0; c < DVT; c += 4)
        *reinterpret_cast<float4*>(dst + c) = make_float4(S[c], S[c + 1], S[c + 2], S[c + 3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TM_COLS);
  }
}

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
bool make_map(CUtensorMap* m, const void* base, int B, int T, int H, int D) {
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

}  // namespace

GDN_DEVICE_ERROR_ACCESSOR(device_error_chunk_tc)

bool chunk_tc_supported(const ChunkArgs& a) {
  return a.dtype == kBF16 && a.semantics == kExact && a.dk == DK && a.dv % DVT == 0 &&
         a.chunk == C && a.T > 0 && encode_fn() != nullptr;
}

cudaError_t launch_chunk_tc(const ChunkArgs& a, cudaStream_t st) {
  if (a.B * a.H == 0 || a.T == 0) return cudaSuccess;
  CUtensorMap mk, mq, mv;
  if (!make_map(&mk, a.k, a.B, a.T, a.H, a.dk) || !make_map(&mq, a.q, a.B, a.T, a.H, a.dk) ||
      !make_map(&mv, a.v, a.B, a.T, a.H, a.dv))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(chunk_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       SMEM_BYTES);
  if (e != cudaSuccess) return e;
  dim3 grid(a.dv / DVT, a.B * a.H);
  chunk_tc_kernel<<<grid, kThreads, SMEM_BYTES, st>>>(
      mk, mq, mv, a.g, a.beta, a.h0, static_cast<__nv_bfloat16*>(a.o), a.hT, a.T, a.H, a.dv);
  return cudaGetLastError();
}

}  // namespace gdn
