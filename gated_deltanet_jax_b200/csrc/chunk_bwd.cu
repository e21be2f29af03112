// Backward of the chunked gated delta rule (exact semantics), fp32 CUDA cores.
//
// The reference has no backward of its own: it relies on JAX autodiff of its
// chunk path (ops.py:238-346).  This computes the gradients of the recurrence
// (ops.py:170-184 with an initial / final state) by reverse-mode
// differentiation through its chunked form, step for step as the oracle's
// chunk_exact_backward:
//
//   forward per chunk (C tokens, in-chunk cumulative gate G, state h entering):
//     A = tril_{-1}(beta_i (K K^T) e^{G_i - G_j}),  T = (I + A)^{-1}
//     X = diag(beta) (V - diag(e^G) K h),  V' = T X
//     P = tril_0((Q K^T) e^{G_i - G_j}),   o = diag(e^G) Q h + P V'
//     h_out = e^{G_C} h + (diag(e^{G_C - G}) K)^T V'
//   backward per chunk, given dO and dh_out:
//     dV' = P^T dO + Kd dh_out,  dX = T^T dV',  dT = dV' X^T,  dA = -T^T dT T^T
//     dh  = e^{G_C} dh_out + Q^T (e^G dO) + K^T dKh,  dKh = -(beta e^G) dX
//     plus the gate terms through e^G, e^{G_i - G_j} and e^{G_C - G}.
//
// One CTA per (b, h, DVT-column tile of the state), internal chunks of CB
// tokens (the exact result does not depend on the chunk length).  Pass 1 runs
// the forward over the chunks and stores the state entering each chunk in the
// workspace; pass 2 walks the chunks in reverse.  Gradients that live in one
// column tile (dv, dh0) are written directly; dq, dk, dbeta and the gate
// gradient sum over all columns, so every tile adds its part into fp32
// accumulators (atomic adds: the order of the tiles' additions, and so the
// last bits, may vary from run to run).  A second kernel converts them,
// sums grouped heads, and turns the gradient of the cumulative gate into that
// of g by a reverse in-chunk cumulative sum.
#include <cstdint>

#include "gdn_common.cuh"
#include "gdn_internal.h"
#include "ptx.cuh"

namespace gdn {

namespace {

constexpr int CB = 32;        // internal chunk length
constexpr int DVT = 32;       // state columns per CTA
constexpr int NTB = 256;      // threads

struct BwdSmem {
  int Q, K, V, dO, H, dH, E, KK, Tm, P, dP, dT, Kh, Qh, X, Vp, dVp, dX, dQ, dK, vec, total;
};

__host__ __device__ inline BwdSmem bwd_layout(int DK) {
  BwdSmem L{};
  int o = 0;
  auto take = [&](int n) { const int r = o; o += (n + 3) & ~3; return r; };
  L.Q = take(CB * DK); L.K = take(CB * DK);
  L.V = take(CB * DVT); L.dO = take(CB * DVT);
  L.H = take(DK * DVT); L.dH = take(DK * DVT);
  L.E = take(CB * CB); L.KK = take(CB * CB); L.Tm = take(CB * CB); L.P = take(CB * CB);
  L.dP = take(CB * CB); L.dT = take(CB * CB);
  L.Kh = take(CB * DVT); L.Qh = take(CB * DVT); L.X = take(CB * DVT); L.Vp = take(CB * DVT);
  L.dVp = take(CB * DVT); L.dX = take(CB * DVT);
  L.dQ = take(CB * DK); L.dK = take(CB * DK);
  L.vec = take(8 * CB);       // G, eG, dec, beta, dG, dbeta, (2 spare)
  L.total = o;
  return L;
}

// out[m][n] (=|+=) alpha * sum_k a(m, k) b(k, n) over an M x N output, all CTA threads.
// a(m,k) = TA ? A[k*lda + m] : A[m*lda + k];  b(k,n) = TB ? B[n*ldb + k] : B[k*ldb + n].
template <bool TA, bool TB>
__device__ __forceinline__ void smm(float* out, int ldo, const float* A, int lda, const float* B,
                                    int ldb, int M, int N, int K, float alpha, bool acc) {
  for (int e = threadIdx.x; e < M * N; e += NTB) {
    const int m = e / N, n = e - m * N;
    float s = 0.f;
    for (int kk = 0; kk < K; ++kk) {
      const float a = TA ? A[kk * lda + m] : A[m * lda + kk];
      const float b = TB ? B[n * ldb + kk] : B[kk * ldb + n];
      s = fmaf(a, b, s);
    }
    out[m * ldo + n] = acc ? fmaf(alpha, s, out[m * ldo + n]) : alpha * s;
  }
}

template <typename Tin>
__device__ __forceinline__ float ld(const Tin* p, size_t i) { return to_f32(p[i]); }

// Everything of chunk n that both passes need, recomputed from the inputs and
// the state entering the chunk (in smem H): G, e^G, e^{G_C - G}, beta, E, KK,
// T = (I + A)^{-1}, Kh = K h, X, V' = T X.  Returns e^{G_C}.
template <typename Tin>
__device__ float chunk_forward(float* sm, const BwdSmem& L, const Tin* q, const Tin* k,
                               const Tin* v, const float* g, const float* beta, size_t row0,
                               int t0, int T, int H, int Hk, int h, int DK, int dv, int c0,
                               bool need_q) {
  const int tid = threadIdx.x;
  float* sQ = sm + L.Q; float* sK = sm + L.K; float* sV = sm + L.V;
  float* sG = sm + L.vec; float* seG = sG + CB; float* sdec = sG + 2 * CB; float* sb = sG + 3 * CB;
  const int hq = h * Hk / H;
  for (int e = tid; e < CB * DK; e += NTB) {
    const int i = e / DK, d = e - i * DK, t = t0 + i;
    const size_t off = ((row0 + t) * Hk + hq) * DK + d;
    sK[e] = t < T ? ld(k, off) : 0.f;
    if (need_q) sQ[e] = t < T ? ld(q, off) : 0.f;
  }
  for (int e = tid; e < CB * DVT; e += NTB) {
    const int i = e / DVT, c = e - i * DVT, t = t0 + i;
    sV[e] = t < T ? ld(v, ((row0 + t) * H + h) * dv + c0 + c) : 0.f;
  }
  if (tid < 32) {
    // in-chunk inclusive cumulative gate (CB == 32: one token per lane)
    const int t = t0 + tid;
    const size_t off = (row0 + t) * H + h;
    const float gi = t < T ? g[off] : 0.f;
    float incl = gi;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, incl, o);
      if (tid >= o) incl += y;
    }
    const float GC = __shfl_sync(0xffffffffu, incl, 31);
    sG[tid] = incl;
    seG[tid] = __expf(incl);
    sdec[tid] = __expf(GC - incl);
    sb[tid] = t < T ? beta[off] : 0.f;
  }
  __syncthreads();
  float* sE = sm + L.E; float* sKK = sm + L.KK; float* sT = sm + L.Tm;
  for (int e = tid; e < CB * CB; e += NTB) {
    const int i = e / CB, j = e - i * CB;
    sE[e] = j <= i ? __expf(sG[i] - sG[j]) : 0.f;
  }
  smm<false, true>(sKK, CB, sK, DK, sK, DK, CB, CB, DK, 1.f, false);   // K K^T
  __syncthreads();
  // A (strictly lower) into dT as scratch, then T = (I + A)^{-1} by substitution
  float* sA = sm + L.dT;
  for (int e = tid; e < CB * CB; e += NTB) {
    const int i = e / CB, j = e - i * CB;
    sA[e] = j < i ? sb[i] * sKK[e] * sE[e] : 0.f;
  }
  __syncthreads();
  if (tid < CB) {
    const int c = tid;
    for (int r = 0; r < CB; ++r) {
      float s = (r == c) ? 1.f : 0.f;
      for (int j = c; j < r; ++j) s = fmaf(-sA[r * CB + j], sT[j * CB + c], s);
      sT[r * CB + c] = r < c ? 0.f : s;
    }
  }
  // Kh = K h
  float* sKh = sm + L.Kh; float* sH = sm + L.H;
  smm<false, false>(sKh, DVT, sK, DK, sH, DVT, CB, DVT, DK, 1.f, false);
  __syncthreads();
  float* sX = sm + L.X;
  for (int e = tid; e < CB * DVT; e += NTB) {
    const int i = e / DVT;
    sX[e] = sb[i] * (sV[e] - seG[i] * sKh[e]);
  }
  __syncthreads();
  smm<false, false>(sm + L.Vp, DVT, sT, CB, sX, DVT, CB, DVT, CB, 1.f, false);   // V' = T X
  __syncthreads();
  return seG[CB - 1];
}

template <typename Tin>
__global__ void __launch_bounds__(NTB)
chunk_bwd_kernel(const Tin* __restrict__ q, const Tin* __restrict__ k, const Tin* __restrict__ v,
                 const float* __restrict__ g, const float* __restrict__ beta,
                 const float* __restrict__ h0, const Tin* __restrict__ dO,
                 const float* __restrict__ dhT, Tin* __restrict__ dv_out,
                 float* __restrict__ dh0, float* __restrict__ states, float* __restrict__ acc_dq,
                 float* __restrict__ acc_dk, float* __restrict__ acc_db,
                 float* __restrict__ acc_dG, int T, int H, int Hk, int DK, int dv) {
  extern __shared__ float sm[];
  const BwdSmem L = bwd_layout(DK);
  const int tid = threadIdx.x;
  const int bh = blockIdx.y, b = bh / H, h = bh - b * H;
  const int c0 = blockIdx.x * DVT;
  const int N = (T + CB - 1) / CB;
  const size_t row0 = (size_t)b * T;
  float* sH = sm + L.H; float* sdH = sm + L.dH;
  float* sK = sm + L.K; float* sQ = sm + L.Q; float* sV = sm + L.V; float* sdO = sm + L.dO;
  float* sG = sm + L.vec; float* seG = sG + CB; float* sdec = sG + 2 * CB; float* sb = sG + 3 * CB;
  float* sdG = sG + 4 * CB; float* sdb = sG + 5 * CB;

  // ---- pass 1: forward, storing the state entering every chunk ----
  for (int e = tid; e < DK * DVT; e += NTB) {
    const int r = e / DVT, c = e - r * DVT;
    sH[e] = h0 ? h0[((size_t)bh * DK + r) * dv + c0 + c] : 0.f;
  }
  __syncthreads();
  for (int n = 0; n < N; ++n) {
    for (int e = tid; e < DK * DVT; e += NTB) {
      const int r = e / DVT, c = e - r * DVT;
      states[(((size_t)bh * N + n) * DK + r) * dv + c0 + c] = sH[e];
    }
    const float eGC = chunk_forward(sm, L, q, k, v, g, beta, row0, n * CB, T, H, Hk, h, DK, dv,
                                    c0, false);
    // h <- e^{G_C} h + Kd^T V'
    const float* sVp = sm + L.Vp;
    for (int e = tid; e < DK * DVT; e += NTB) {
      const int d = e / DVT, c = e - d * DVT;
      float s = 0.f;
      for (int i = 0; i < CB; ++i) s = fmaf(sdec[i] * sK[i * DK + d], sVp[i * DVT + c], s);
      sH[e] = fmaf(eGC, sH[e], s);
    }
    __syncthreads();
  }

  // ---- pass 2: reverse ----
  for (int e = tid; e < DK * DVT; e += NTB) {
    const int r = e / DVT, c = e - r * DVT;
    sdH[e] = dhT ? dhT[((size_t)bh * DK + r) * dv + c0 + c] : 0.f;
  }
  __syncthreads();
  for (int n = N - 1; n >= 0; --n) {
    const int t0 = n * CB;
    for (int e = tid; e < DK * DVT; e += NTB) {
      const int r = e / DVT, c = e - r * DVT;
      sH[e] = states[(((size_t)bh * N + n) * DK + r) * dv + c0 + c];
    }
    for (int e = tid; e < CB * DVT; e += NTB) {
      const int i = e / DVT, c = e - i * DVT, t = t0 + i;
      sdO[e] = t < T ? ld(dO, ((row0 + t) * H + h) * dv + c0 + c) : 0.f;
    }
    __syncthreads();
    const float eGC = chunk_forward(sm, L, q, k, v, g, beta, row0, t0, T, H, Hk, h, DK, dv, c0,
                                    true);
    float* sE = sm + L.E; float* sKK = sm + L.KK; float* sT = sm + L.Tm; float* sP = sm + L.P;
    float* sdP = sm + L.dP; float* sdT = sm + L.dT;
    float* sKh = sm + L.Kh; float* sQh = sm + L.Qh; float* sX = sm + L.X; float* sVp = sm + L.Vp;
    float* sdVp = sm + L.dVp; float* sdX = sm + L.dX;
    float* sdQ = sm + L.dQ; float* sdK = sm + L.dK;
    // P, Qh
    smm<false, true>(sP, CB, sQ, DK, sK, DK, CB, CB, DK, 1.f, false);
    smm<false, false>(sQh, DVT, sQ, DK, sH, DVT, CB, DVT, DK, 1.f, false);
    __syncthreads();
    for (int e = tid; e < CB * CB; e += NTB) sP[e] *= sE[e];   // E is 0 above the diagonal
    if (tid < CB) { sdG[tid] = 0.f; sdb[tid] = 0.f; }
    __syncthreads();
    // dV' = Kd dh_out + P^T dO
    for (int e = tid; e < CB * DVT; e += NTB) {
      const int i = e / DVT, c = e - i * DVT;
      float s = 0.f;
      for (int d = 0; d < DK; ++d) s = fmaf(sK[i * DK + d], sdH[d * DVT + c], s);
      float s2 = 0.f;
      for (int j = 0; j < CB; ++j) s2 = fmaf(sP[j * CB + i], sdO[j * DVT + c], s2);
      sdVp[e] = fmaf(sdec[i], s, s2);
    }
    // dQ = e^G (dO h^T) ; dK = dec (V' dh_out^T)   (partials of this tile)
    for (int e = tid; e < CB * DK; e += NTB) {
      const int i = e / DK, d = e - i * DK;
      float sq = 0.f, sk = 0.f;
      for (int c = 0; c < DVT; ++c) {
        sq = fmaf(sdO[i * DVT + c], sH[d * DVT + c], sq);
        sk = fmaf(sVp[i * DVT + c], sdH[d * DVT + c], sk);
      }
      sdQ[e] = seG[i] * sq;
      sdK[e] = sdec[i] * sk;
    }
    // dP = causal(dO V'^T);  dT = dV' X^T (after dV' is complete)
    __syncthreads();
    smm<false, true>(sdP, CB, sdO, DVT, sVp, DVT, CB, CB, DVT, 1.f, false);
    smm<false, true>(sdT, CB, sdVp, DVT, sX, DVT, CB, CB, DVT, 1.f, false);
    __syncthreads();
    // gate terms: dG_C (e^{G_C}<h, dh_out> + sum_i <dKd_i, Kd_i>), -<dKd_i, Kd_i>,
    // e^{G_i} <dO_i, Qh_i>, row/column sums of dP * P.  dG_C goes to the last real
    // token of the chunk (padding carries no other gate gradient, so the reverse
    // cumulative sum is the same as from the padded end).
    const int last = min(CB, T - t0) - 1;
    if (tid < 32) {
      float part = 0.f;
      for (int e = tid; e < DK * DVT; e += 32) part = fmaf(sH[e], sdH[e], part);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      if (tid == 0) atomicAdd(&sdG[last], eGC * part);
    }
    if (tid >= 32 && tid < 32 + CB) {
      const int i = tid - 32;
      // <dKd_i, Kd_i> = dec_i * <V'_i dh_out^T, K_i> ... = sum_d dK_i,d(before dec) * dec_i K_i,d
      float kd = 0.f;
      for (int d = 0; d < DK; ++d) kd = fmaf(sdK[i * DK + d], sK[i * DK + d], kd);
      // sdK holds dec_i * (V' dh^T)_i, so <dKd_i, Kd_i> = kd
      float oq = 0.f;
      for (int c = 0; c < DVT; ++c) oq = fmaf(sdO[i * DVT + c], sQh[i * DVT + c], oq);
      float pp = 0.f;
      for (int j = 0; j <= i; ++j) pp = fmaf(sdP[i * CB + j], sP[i * CB + j], pp);
      for (int j = i; j < CB; ++j) pp = fmaf(-sdP[j * CB + i], sP[j * CB + i], pp);
      atomicAdd(&sdG[i], seG[i] * oq + pp - kd);
      atomicAdd(&sdG[last], kd);
    }
    __syncthreads();
    // dQ += (dP*E) K ; dK += (dP*E)^T Q   (dP*E formed in place: E = 0 above the diagonal)
    for (int e = tid; e < CB * CB; e += NTB) sdP[e] *= sE[e];
    __syncthreads();
    smm<false, false>(sdQ, DK, sdP, CB, sK, DK, CB, DK, CB, 1.f, true);
    smm<true, false>(sdK, DK, sdP, CB, sQ, DK, CB, DK, CB, 1.f, true);
    // dX = T^T dV'
    smm<true, false>(sdX, DVT, sT, CB, sdVp, DVT, CB, DVT, CB, 1.f, false);
    __syncthreads();
    // dA = -T^T dT T^T (strictly lower), into dP (free now)
    smm<true, false>(sdP, CB, sT, CB, sdT, CB, CB, CB, CB, 1.f, false);   // T^T dT
    __syncthreads();
    smm<false, true>(sdT, CB, sdP, CB, sT, CB, CB, CB, CB, -1.f, false);  // (T^T dT) T^T
    __syncthreads();
    for (int e = tid; e < CB * CB; e += NTB) {
      const int i = e / CB, j = e - i * CB;
      if (j >= i) sdT[e] = 0.f;                                          // dA
    }
    // dV (this tile, direct), dbeta, dKh = -(beta e^G) dX, gate term <dKh, Kh>
    for (int e = tid; e < CB * DVT; e += NTB) {
      const int i = e / DVT, c = e - i * DVT, t = t0 + i;
      if (t < T)
        dv_out[((row0 + t) * H + h) * dv + c0 + c] = from_f32<Tin>(sb[i] * sdX[e]);
    }
    __syncthreads();
    if (tid < CB) {
      const int i = tid;
      float db = 0.f, gk = 0.f;
      for (int c = 0; c < DVT; ++c) {
        const float dx = sdX[i * DVT + c], kh = sKh[i * DVT + c];
        db = fmaf(dx, sV[i * DVT + c] - seG[i] * kh, db);
        gk = fmaf(-sb[i] * seG[i] * dx, kh, gk);
      }
      sdb[i] += db;
      sdG[i] += gk;
    }
    // dKh into dX (scaled in place)
    __syncthreads();
    for (int e = tid; e < CB * DVT; e += NTB) {
      const int i = e / DVT;
      sdX[e] *= -sb[i] * seG[i];
    }
    __syncthreads();
    // dK += dKh h^T
    smm<false, true>(sdK, DK, sdX, DVT, sH, DVT, CB, DK, DVT, 1.f, true);
    // A-terms: dAE = dA * E;  dbeta_i += sum_j dAE_ij KK_ij;  dG from dA * A
    for (int e = tid; e < CB * CB; e += NTB) sdP[e] = sdT[e] * sE[e];   // dAE
    __syncthreads();
    if (tid < CB) {
      const int i = tid;
      float db = 0.f, ga = 0.f;
      for (int j = 0; j < i; ++j) {
        const float a = sb[i] * sKK[i * CB + j] * sE[i * CB + j];
        db = fmaf(sdP[i * CB + j], sKK[i * CB + j], db);
        ga = fmaf(sdT[i * CB + j], a, ga);
      }
      for (int j = i + 1; j < CB; ++j) {
        const float a = sb[j] * sKK[j * CB + i] * sE[j * CB + i];
        ga = fmaf(-sdT[j * CB + i], a, ga);
      }
      sdb[i] += db;
      sdG[i] += ga;
    }
    // dK += diag(beta) dAE K + dAE^T diag(beta) K
    for (int e = tid; e < CB * DK; e += NTB) {
      const int i = e / DK, d = e - i * DK;
      float s1 = 0.f, s2 = 0.f;
      for (int j = 0; j < CB; ++j) {
        s1 = fmaf(sdP[i * CB + j], sK[j * DK + d], s1);
        s2 = fmaf(sdP[j * CB + i], sb[j] * sK[j * DK + d], s2);
      }
      sdK[e] += sb[i] * s1 + s2;
    }
    __syncthreads();
    // dh <- e^{G_C} dh_out + Q^T (e^G dO) + K^T dKh
    for (int e = tid; e < DK * DVT; e += NTB) {
      const int d = e / DVT, c = e - d * DVT;
      float s = 0.f;
      for (int i = 0; i < CB; ++i)
        s = fmaf(sQ[i * DK + d], seG[i] * sdO[i * DVT + c], fmaf(sK[i * DK + d], sdX[i * DVT + c], s));
      sdH[e] = fmaf(eGC, sdH[e], s);
    }
    // this tile's parts of dq, dk, dbeta and the cumulative-gate gradient
    for (int e = tid; e < CB * DK; e += NTB) {
      const int i = e / DK, d = e - i * DK, t = t0 + i;
      if (t < T) {
        const size_t off = ((row0 + t) * H + h) * DK + d;
        atomicAdd(&acc_dq[off], sdQ[e]);
        atomicAdd(&acc_dk[off], sdK[e]);
      }
    }
    if (tid < CB && t0 + tid < T) {
      const size_t off = (row0 + t0 + tid) * H + h;
      atomicAdd(&acc_db[off], sdb[tid]);
      atomicAdd(&acc_dG[off], sdG[tid]);
    }
    __syncthreads();
  }
  for (int e = tid; e < DK * DVT; e += NTB) {
    const int r = e / DVT, c = e - r * DVT;
    if (dh0) dh0[((size_t)bh * DK + r) * dv + c0 + c] = sdH[e];
  }
}

// dq, dk in the input dtype (value heads of a group summed into their q/k
// head), dbeta, and dg = reverse in-chunk cumulative sum of the gradient of G.
template <typename Tin>
__global__ void chunk_bwd_finish_kernel(const float* __restrict__ acc_dq,
                                        const float* __restrict__ acc_dk,
                                        const float* __restrict__ acc_db,
                                        const float* __restrict__ acc_dG, Tin* __restrict__ dq,
                                        Tin* __restrict__ dk, float* __restrict__ dg,
                                        float* __restrict__ dbeta, int B, int T, int H, int Hk,
                                        int DK) {
  const int rep = H / Hk;
  const size_t nqk = (size_t)B * T * Hk * DK;
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < nqk;
       e += (size_t)gridDim.x * blockDim.x) {
    const int d = (int)(e % DK);
    const size_t r = e / DK;                 // (b, t, hk)
    const int hk = (int)(r % Hk);
    const size_t bt = r / Hk;
    float sq = 0.f, sk = 0.f;
    for (int j = 0; j < rep; ++j) {
      const size_t off = (bt * H + (size_t)hk * rep + j) * DK + d;
      sq += acc_dq[off];
      sk += acc_dk[off];
    }
    dq[e] = from_f32<Tin>(sq);
    dk[e] = from_f32<Tin>(sk);
  }
  const size_t nseg = (size_t)B * H * ((T + CB - 1) / CB);
  for (size_t s = blockIdx.x * (size_t)blockDim.x + threadIdx.x; s < nseg;
       s += (size_t)gridDim.x * blockDim.x) {
    const int nch = (T + CB - 1) / CB;
    const int n = (int)(s % nch);
    const size_t bhh = s / nch;
    const int h = (int)(bhh % H);
    const size_t b = bhh / H;
    float run = 0.f;
    const int t_end = min(T, (n + 1) * CB);
    for (int t = t_end - 1; t >= n * CB; --t) {
      const size_t off = (b * T + t) * H + h;
      run += acc_dG[off];
      dg[off] = run;
      dbeta[off] = acc_db[off];
    }
  }
}

template <typename Tin>
cudaError_t launch_bwd_t(const ChunkBwdArgs& a, cudaStream_t st) {
  const BwdSmem L = bwd_layout(a.dk);
  const size_t smem = (size_t)L.total * sizeof(float);
  auto kern = chunk_bwd_kernel<Tin>;
  static std::atomic<int> smem_set[kMaxDevices] = {};
  cudaError_t e = ensure_smem(kern, (int)smem, smem_set);
  if (e != cudaSuccess) return e;
  float* ws = static_cast<float*>(a.workspace);
  const int N = (a.T + CB - 1) / CB;
  const size_t n_states = (size_t)a.B * a.H * N * a.dk * a.dv;
  const size_t n_qk = (size_t)a.B * a.T * a.H * a.dk;
  const size_t n_tok = (size_t)a.B * a.T * a.H;
  float* states = ws;
  float* acc_dq = states + n_states;
  float* acc_dk = acc_dq + n_qk;
  float* acc_db = acc_dk + n_qk;
  float* acc_dG = acc_db + n_tok;
  e = cudaMemsetAsync(acc_dq, 0, sizeof(float) * (2 * n_qk + 2 * n_tok), st);
  if (e != cudaSuccess) return e;
  dim3 grid(a.dv / DVT, a.B * a.H);
  kern<<<grid, NTB, smem, st>>>(
      static_cast<const Tin*>(a.q), static_cast<const Tin*>(a.k), static_cast<const Tin*>(a.v),
      a.g, a.beta, a.h0, static_cast<const Tin*>(a.dO), a.dhT, static_cast<Tin*>(a.dv_out),
      a.dh0, states, acc_dq, acc_dk, acc_db, acc_dG, a.T, a.H, a.Hk, a.dk, a.dv);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const size_t work = n_qk > n_tok ? n_qk : n_tok;
  const int blocks = (int)((work + 255) / 256 < 8 * 148 ? (work + 255) / 256 : 8 * 148);
  chunk_bwd_finish_kernel<Tin><<<blocks, 256, 0, st>>>(
      acc_dq, acc_dk, acc_db, acc_dG, static_cast<Tin*>(a.dq), static_cast<Tin*>(a.dk_out),
      a.dg, a.dbeta, a.B, a.T, a.H, a.Hk, a.dk);
  return cudaGetLastError();
}

}  // namespace

size_t chunk_bwd_workspace_bytes(int B, int T, int H, int dk, int dv) {
  const size_t N = (size_t)((T + CB - 1) / CB);
  return sizeof(float) * ((size_t)B * H * N * dk * dv + 2 * (size_t)B * T * H * dk +
                          2 * (size_t)B * T * H);
}

bool chunk_bwd_supported(const ChunkBwdArgs& a) {
  return a.dv % DVT == 0 && (size_t)bwd_layout(a.dk).total * sizeof(float) <= 200 * 1024;
}

cudaError_t launch_chunk_bwd(const ChunkBwdArgs& a, cudaStream_t st) {
  if (a.B * a.H == 0 || a.T == 0) return cudaSuccess;
  return a.dtype == kBF16 ? launch_bwd_t<__nv_bfloat16>(a, st) : launch_bwd_t<float>(a, st);
}

}  // namespace gdn
