// Device helpers shared by the tensor-core chunk kernels (chunk_tc.cu,
// chunk_scan.cu): bf16 packing, the in-chunk gate vectors, and the solve of
// T = (I + A)^{-1} for one chunk of 64 tokens (16x16 diagonal blocks by
// substitution, off-diagonal blocks on tf32 warp MMAs).
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "gdn_common.cuh"
#include "ptx.cuh"

namespace gdn {
namespace {

constexpr int C = 64;    // tokens per chunk
constexpr int LDF = 68;  // fp32 row stride of the A / T matrices (16-byte aligned rows)

constexpr uint32_t IDESC_KK = idesc_bf16(128, 64, 0, 0);  // A K-major, B K-major
constexpr uint32_t IDESC_KM = idesc_bf16(128, 64, 0, 1);  // A K-major, B MN-major
constexpr uint32_t IDESC_MM = idesc_bf16(128, 64, 1, 1);  // A MN-major, B MN-major
constexpr uint32_t SW128 = 2;

// Gate vectors of one chunk (C tokens, in-chunk inclusive cumulative gate G).
struct VecBuf {
  float G[C], eG[C], dec[C], beta[C];
  float F[C][4];  // e^{G_i - G_{16k}} for k <= i / 16 (gate factors, row part)
  float E[C];     // e^{G_{16 floor(j/16)} - G_j}      (gate factors, column part)
  float eGC;
  int direct;     // 1: a factor exponent exceeds 40; form e^{G_i - G_j} directly
  float pad[2];
};

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

// fp32 value rounded to tf32 (kept as an fp32 bit pattern with the low 13 bits clear).
__device__ __forceinline__ float rtf32(float x) { return __uint_as_float(to_tf32(x)); }

// Warp-level 16x16 block products for the triangular solve (tf32 m16n8k8,
// fp32 accumulate).  Operands are read as stored: every value in the solve
// scratch is already rounded to tf32.  acc holds the C fragments of the two
// 16x8 halves: thread (g = lane/4, t = lane%4) owns rows g, g+8 and columns
// 2t, 2t+1 of each.
__device__ __forceinline__ void mma16x16(float (&acc)[2][4], const float* A, int lda,
                                         const float* B, int ldb, int gq, int tq) {
#pragma unroll
  for (int kk = 0; kk < 16; kk += 8) {
    const uint32_t a[4] = {__float_as_uint(A[gq * lda + kk + tq]),
                           __float_as_uint(A[(gq + 8) * lda + kk + tq]),
                           __float_as_uint(A[gq * lda + kk + tq + 4]),
                           __float_as_uint(A[(gq + 8) * lda + kk + tq + 4])};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const uint32_t bb[2] = {__float_as_uint(B[(kk + tq) * ldb + nt * 8 + gq]),
                              __float_as_uint(B[(kk + tq + 4) * ldb + nt * 8 + gq])};
      mma_tf32(acc[nt], a, bb);
    }
  }
}

__device__ __forceinline__ void store16x16(float* D, int ld, const float (&acc)[2][4], float s,
                                           int gq, int tq) {
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    *reinterpret_cast<float2*>(D + gq * ld + nt * 8 + 2 * tq) =
        make_float2(rtf32(s * acc[nt][0]), rtf32(s * acc[nt][1]));
    *reinterpret_cast<float2*>(D + (gq + 8) * ld + nt * 8 + 2 * tq) =
        make_float2(rtf32(s * acc[nt][2]), rtf32(s * acc[nt][3]));
  }
}

__device__ __forceinline__ void load16x16(float (&acc)[2][4], const float* D, int ld, float s,
                                          int gq, int tq) {
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    const float2 x = *reinterpret_cast<const float2*>(D + gq * ld + nt * 8 + 2 * tq);
    const float2 y = *reinterpret_cast<const float2*>(D + (gq + 8) * ld + nt * 8 + 2 * tq);
    acc[nt][0] = s * x.x; acc[nt][1] = s * x.y; acc[nt][2] = s * y.x; acc[nt][3] = s * y.y;
  }
}

// Off-diagonal blocks of T = (I + A)^{-1} (4x4 blocks of 16; T_ii known from the
// diagonal substitution).  With M_xy = A_xy T_yy the block recurrences
//   T_x,x-1 = -T_xx M_x,x-1
//   T_20 = T_22 (M_21 M_10 - M_20)             = T_22 N_20
//   T_31 = T_33 (M_32 M_21 - M_31)             = T_33 N_31
//   T_30 = T_33 (M_31 M_10 - M_30) + T_32 N_20 = T_33 N_30 + T_32 N_20
// need three dependent product steps:
//   phase 0: M_10 M_20 M_30 M_21 M_31 M_32
//   phase 1: T_10 T_21 T_32, N_20 N_30 N_31
//   phase 2: T_20 T_31 T_30
// Intermediates live in the fp32 T scratch: the M blocks in its (unused) strictly
// upper blocks, N_20 N_30 N_31 and T_32 in lower blocks whose fp32 values are
// never needed (finished T blocks go straight to the bf16 tile).
// One word per warp task, one byte per field: A1, B1, A2, B2 (second product
// or -1), C (subtracted, or -1), fp32 destination, bf16 tile block (or -1),
// output sign.  Block codes: 16 * (0 = A scratch, 1 = T scratch) + 4 *
// block_row + block_col.
constexpr uint64_t solve_task(int a1, int b1, int a2, int b2, int c, int d, int blk, int sc) {
  return (uint64_t)(uint8_t)a1 | (uint64_t)(uint8_t)b1 << 8 | (uint64_t)(uint8_t)a2 << 16 |
         (uint64_t)(uint8_t)b2 << 24 | (uint64_t)(uint8_t)c << 32 | (uint64_t)(uint8_t)d << 40 |
         (uint64_t)(uint8_t)blk << 48 | (uint64_t)(uint8_t)sc << 56;
}
__device__ __forceinline__ int task_field(uint64_t t, int k) {
  return (int)(signed char)(uint8_t)(t >> (8 * k));
}
constexpr uint64_t kNoTask = solve_task(-1, -1, -1, -1, -1, -1, -1, 0);
#define SA(i, j) ((i) * 4 + (j))
#define ST(i, j) (16 + (i) * 4 + (j))
__constant__ uint64_t kSolveTask[3][6] = {
    {solve_task(SA(1, 0), ST(0, 0), -1, -1, -1, ST(0, 1), -1, 1),
     solve_task(SA(2, 0), ST(0, 0), -1, -1, -1, ST(0, 2), -1, 1),
     solve_task(SA(3, 0), ST(0, 0), -1, -1, -1, ST(0, 3), -1, 1),
     solve_task(SA(2, 1), ST(1, 1), -1, -1, -1, ST(1, 2), -1, 1),
     solve_task(SA(3, 1), ST(1, 1), -1, -1, -1, ST(1, 3), -1, 1),
     solve_task(SA(3, 2), ST(2, 2), -1, -1, -1, ST(2, 3), -1, 1)},
    {solve_task(ST(1, 1), ST(0, 1), -1, -1, -1, -1, SA(1, 0), -1),
     solve_task(ST(2, 2), ST(1, 2), -1, -1, -1, -1, SA(2, 1), -1),
     solve_task(ST(3, 3), ST(2, 3), -1, -1, -1, ST(3, 2), SA(3, 2), -1),
     solve_task(ST(1, 2), ST(0, 1), -1, -1, ST(0, 2), ST(1, 0), -1, 1),
     solve_task(ST(1, 3), ST(0, 1), -1, -1, ST(0, 3), ST(2, 0), -1, 1),
     solve_task(ST(2, 3), ST(1, 2), -1, -1, ST(1, 3), ST(2, 1), -1, 1)},
    {solve_task(ST(2, 2), ST(1, 0), -1, -1, -1, -1, SA(2, 0), 1),
     solve_task(ST(3, 3), ST(2, 1), -1, -1, -1, -1, SA(3, 1), 1),
     solve_task(ST(3, 3), ST(2, 0), ST(3, 2), ST(1, 0), -1, -1, SA(3, 0), 1), kNoTask, kNoTask,
     kNoTask},
};
#undef SA
#undef ST

// s * acc as bf16 into the 16x16 block at (r0, c0) of a 128-byte-swizzled tile.
__device__ __forceinline__ void store16x16_bf16(unsigned char* tile, int r0, int c0,
                                                const float (&acc)[2][4], float s, int gq,
                                                int tq) {
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    const int col = c0 + nt * 8 + 2 * tq;
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      const int row = r0 + gq + 8 * h2;
      *reinterpret_cast<__nv_bfloat162*>(tile + sw128(row, col >> 3) + (col & 7) * 2) =
          __floats2bfloat162_rn(s * acc[nt][2 * h2], s * acc[nt][2 * h2 + 1]);
    }
  }
}

__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Named barrier that also ANDs a predicate over its `nthreads` threads: every
// thread returns true only if all of them passed true.
__device__ __forceinline__ bool named_sync_and(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}


// s * acc * rs[row] as bf16 into the 16x16 block at (r0, c0) of a
// 128-byte-swizzled tile (rows scaled by the fp32 vector rs).
__device__ __forceinline__ void store16x16_bf16_rows(unsigned char* tile, int r0, int c0,
                                                     const float (&acc)[2][4], float s,
                                                     const float* rs, int gq, int tq) {
#pragma unroll
  for (int h2 = 0; h2 < 2; ++h2) {
    const int row = r0 + gq + 8 * h2;
    const float sr = s * rs[row];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int col = c0 + nt * 8 + 2 * tq;
      *reinterpret_cast<__nv_bfloat162*>(tile + sw128(row, col >> 3) + (col & 7) * 2) =
          __floats2bfloat162_rn(sr * acc[nt][2 * h2], sr * acc[nt][2 * h2 + 1]);
    }
  }
}

// Gate vectors of one chunk, by one warp (lane l holds tokens 2l, 2l + 1: g0,
// g1 and beta b0, b1; zero past the sequence).  G is the in-chunk inclusive
// cumulative gate; eG = e^G, dec = e^{G_C - G}, eGC = e^{G_C}.  With
// `factors`, also the separable factors e^{G_i - G_j} = F[i][j/16] * E[j]
// (j <= i): every factor exponent lies inside one 16-token block or runs from
// a block start to a later row; if any exceeds 40 (a factor could overflow,
// or hide a non-negligible product behind an underflowed partner) the chunk
// is flagged to form e^{G_i - G_j} directly.
__device__ __forceinline__ void chunk_gate_vectors(VecBuf& vb, float g0, float g1, float b0,
                                                   float b1, bool factors, int lane) {
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
  vb.beta[2 * lane] = b0;
  vb.beta[2 * lane + 1] = b1;
  vb.eG[2 * lane] = gate_exp(G0);
  vb.eG[2 * lane + 1] = gate_exp(G1);
  vb.dec[2 * lane] = gate_exp(GC - G0);
  vb.dec[2 * lane + 1] = gate_exp(GC - G1);
  if (lane == 0) vb.eGC = gate_exp(GC);
  __syncwarp();
  float big = 0.f;
#pragma unroll 1
  for (int half = 0; half < (factors ? 2 : 0); ++half) {
    const int i = lane + 32 * half;
    const float Gi = vb.G[i];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float x = (16 * k <= i) ? Gi - vb.G[16 * k] : 0.f;
      vb.F[i][k] = gate_exp(x);
      big = fmaxf(big, x);
    }
    const float x = vb.G[i & ~15] - Gi;
    vb.E[i] = gate_exp(x);
    big = fmaxf(big, x);
  }
  const int direct = __any_sync(0xffffffffu, big > 40.f) ? 1 : 0;
  if (lane == 0) vb.direct = direct;
  __syncwarp();
}

// T = (I + A)^{-1}, step 1, from shared memory: the four 16x16 diagonal
// blocks by column-oriented substitution, one thread (pi < 64) per column of a
// block; the dependent chain is 15 FMAs long, and A is read four columns at a
// time.  Writes the blocks to the fp32 scratch TF (rounded to tf32) and as
// bf16 into rows 0-63 of the swizzled tile tpt; with tdt, also
// e^{G_C - G_i} T_ij (row-scaled by dec) as bf16 into tdt.
__device__ __forceinline__ void solve_diag(const float* AF, float* TF, unsigned char* tpt,
                                           unsigned char* tdt, const float* dec, int pi) {
  const int blk = pi >> 4, c = pi & 15;
  const float* Ab = AF + (blk * 16) * LDF + blk * 16;
  float t[16];
#pragma unroll
  for (int r = 0; r < 16; ++r) t[r] = (r == c) ? 1.f : 0.f;
#pragma unroll
  for (int j0 = 0; j0 < 16; j0 += 4) {
    float a4[16][4];
#pragma unroll
    for (int r = j0 + 1; r < 16; ++r) {
      const float4 x = *reinterpret_cast<const float4*>(Ab + r * LDF + j0);
      a4[r][0] = x.x; a4[r][1] = x.y; a4[r][2] = x.z; a4[r][3] = x.w;
    }
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
#pragma unroll
      for (int r = j0 + jj + 1; r < 16; ++r) t[r] = fmaf(-a4[r][jj], t[j0 + jj], t[r]);
    }
  }
  float* Tb = TF + (blk * 16) * LDF + blk * 16;
#pragma unroll
  for (int r = 0; r < 16; ++r) {
    Tb[r * LDF + c] = rtf32(t[r]);
    const int row = blk * 16 + r, col = blk * 16 + c;
    const uint32_t off = sw128(row, col >> 3) + (col & 7) * 2;
    *reinterpret_cast<__nv_bfloat16*>(tpt + off) = __float2bfloat16_rn(t[r]);
    if (tdt) *reinterpret_cast<__nv_bfloat16*>(tdt + off) = __float2bfloat16_rn(dec[row] * t[r]);
  }
}

// T = (I + A)^{-1}, step 1, from registers: one half-warp per 16x16 diagonal
// block `blk`, lane r of the half holding row r of the block's strictly lower
// A (arow, tf32-rounded, as in AF).  Row-oriented substitution: once row m of
// the block's inverse is final, every later row subtracts A[r][m] times it,
// with row m's entries (columns 0..m) taken from its lane by shuffles; the
// dependent chain is 15 steps.  Writes the block to TF (tf32-rounded), as bf16
// into tpt and, row-scaled by dec, into tdt.
__device__ __forceinline__ void solve_diag_rows(const float (&arow)[16], int blk, int lane,
                                                float* TF, unsigned char* tpt,
                                                unsigned char* tdt, const float* dec) {
  const int r = lane & 15;
  const int src = lane & 16;
  float t[16];
#pragma unroll
  for (int c = 0; c < 16; ++c) t[c] = (c == r) ? 1.f : 0.f;
#pragma unroll
  for (int m = 0; m < 15; ++m) {
    const float a = r > m ? arow[m] : 0.f;
#pragma unroll
    for (int c = 0; c <= m; ++c) t[c] = fmaf(-a, __shfl_sync(0xffffffffu, t[c], src | m), t[c]);
  }
  const int row = 16 * blk + r;
  float* Tr = TF + row * LDF + 16 * blk;
#pragma unroll
  for (int c = 0; c < 16; c += 4)
    *reinterpret_cast<float4*>(Tr + c) =
        make_float4(rtf32(t[c]), rtf32(t[c + 1]), rtf32(t[c + 2]), rtf32(t[c + 3]));
  *reinterpret_cast<uint4*>(tpt + sw128(row, 2 * blk)) = pack_bf16x8(t);
  *reinterpret_cast<uint4*>(tpt + sw128(row, 2 * blk + 1)) = pack_bf16x8(t + 8);
  const float d = dec[row];
#pragma unroll
  for (int c = 0; c < 16; ++c) t[c] *= d;
  *reinterpret_cast<uint4*>(tdt + sw128(row, 2 * blk)) = pack_bf16x8(t);
  *reinterpret_cast<uint4*>(tdt + sw128(row, 2 * blk + 1)) = pack_bf16x8(t + 8);
}

// T = (I + A)^{-1}, step 2: the off-diagonal 16x16 blocks in three phases of
// independent warp tasks (tf32 warp MMAs), scheduled by kSolveTask; w8 is the
// warp's index 0..7 among the solving warps, which meet on named barrier
// `bar_id` (`nthreads` threads) between phases.  Finished blocks go to tpt
// (and, row-scaled by dec, to tdt) as bf16.
__device__ __forceinline__ void solve_offdiag(float* AF, float* TF, unsigned char* tpt,
                                              unsigned char* tdt, const float* dec, int w8,
                                              int lane, int bar_id, int nthreads) {
  const uint64_t task0 = w8 < 6 ? kSolveTask[0][w8] : kNoTask;
  const uint64_t task1 = w8 < 6 ? kSolveTask[1][w8] : kNoTask;
  const uint64_t task2 = w8 < 6 ? kSolveTask[2][w8] : kNoTask;
  const int gq = lane >> 2, tq = lane & 3;
  auto blk = [&](int code) {
    return (code >= 16 ? TF : AF) + ((code >> 2) & 3) * 16 * LDF + (code & 3) * 16;
  };
#pragma unroll 1
  for (int ph = 0; ph < 3; ++ph) {
    const uint64_t tk = ph == 0 ? task0 : (ph == 1 ? task1 : task2);
    if (task_field(tk, 0) >= 0) {
      float acc[2][4] = {};
      if (task_field(tk, 4) >= 0) load16x16(acc, blk(task_field(tk, 4)), LDF, -1.f, gq, tq);
#pragma unroll 1
      for (int pi2 = 0; pi2 < (task_field(tk, 2) >= 0 ? 2 : 1); ++pi2)
        mma16x16(acc, blk(task_field(tk, 2 * pi2)), LDF, blk(task_field(tk, 2 * pi2 + 1)), LDF,
                 gq, tq);
      const float sc = (float)task_field(tk, 7);
      if (task_field(tk, 5) >= 0) store16x16(blk(task_field(tk, 5)), LDF, acc, sc, gq, tq);
      const int bt = task_field(tk, 6);
      if (bt >= 0) {
        store16x16_bf16(tpt, (bt >> 2) * 16, (bt & 3) * 16, acc, sc, gq, tq);
        if (tdt) store16x16_bf16_rows(tdt, (bt >> 2) * 16, (bt & 3) * 16, acc, sc, dec, gq, tq);
      }
    }
    if (ph < 2) named_sync(bar_id, nthreads);
  }
}

}  // namespace
}  // namespace gdn
