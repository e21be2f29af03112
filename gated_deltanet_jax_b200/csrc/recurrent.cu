// Fused recurrent gated delta rule (decode), sm_100a.
//
// Replaces the reference's Pallas kernel fused_recurrent_kernel_simple
// (ops.py:162-184): per (b, h) and token t with an fp32 state S [dk, dv],
//     S <- e^{g} S;  u = beta (v - k^T S);  S <- S + k u^T;  o = S^T q.
//
// Design (HBM-bound: the fp32 state is read and written once per call):
//   * The dv columns of S evolve independently, so one CTA owns a column tile
//     of CW columns of one (b, h): grid = (dv / CW, B * H).
//   * Each thread owns 4 consecutive columns (one 128-bit access per row) of
//     RPT rows; a warp's row access is a contiguous 4*CW-byte segment, and the
//     thread's state tile stays in registers across all T tokens.
//   * Both column reductions over dk (k^T S and q^T S) come from the same
//     pre-update state:  with alpha = e^{g},
//         u = beta (v - alpha k^T S),   o = alpha q^T S + (q . k) u,
//     so a token needs one pass over the registers, one warp-shuffle
//     reduction and one shared-memory exchange between warps.
//   * State loads/stores use the streaming cache policy (touched once).
#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {

// kGates: g and beta hold the raw a_proj / b_proj outputs, and each token's
// g = -exp(A_log[h]) softplus(a + dt_bias[h]), beta = sigmoid(b) are formed
// here (the layer's prologue, model.py:136-139; the norm runs afterwards).
template <typename Tin, int DK, int CW, int NT, bool kGates>
__global__ void __launch_bounds__(NT)
recurrent_kernel(const Tin* __restrict__ q, const Tin* __restrict__ k,
                 const Tin* __restrict__ v, const float* __restrict__ g,
                 const float* __restrict__ beta, const float* h0,
                 Tin* __restrict__ o, float* hT, int T, int H, int Hk, int dv,
                 const float* __restrict__ A_log, const float* __restrict__ dt_bias) {
  constexpr int LPR = CW / 4;        // threads across one row of the tile
  constexpr int RPP = NT / LPR;      // rows covered per pass of the CTA
  constexpr int RPT = DK / RPP;      // rows per thread
  constexpr int NWARP = NT / 32;
  static_assert(CW % 4 == 0 && NT % LPR == 0 && DK % RPP == 0 && RPT >= 1, "tile");
  static_assert(LPR <= 32, "a row must fit in one warp");

  __shared__ float s_k[2][DK];
  __shared__ float s_q[2][DK];
  __shared__ float4 s_red[2][NWARP][2][LPR];  // per-warp column partials (k^T S, q^T S)
  __shared__ float s_qk[2][NWARP];

  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int cg = tid % LPR;          // column group (4 columns)
  const int rb = tid / LPR;          // first row
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh - b * H;
  const int hq = h * Hk / H;         // q/k head of this value head (grouped heads)
  const int col = blockIdx.x * CW + cg * 4;

  const size_t sbase = (size_t)bh * DK * dv + col;
  const float negA = kGates ? -expf(A_log[h]) : 0.f;
  const float dtb = kGates ? dt_bias[h] : 0.f;
  float4 S[RPT];
  if (h0 != nullptr) {
#pragma unroll
    for (int i = 0; i < RPT; ++i) S[i] = load4_stream(h0 + sbase + (size_t)(rb + i * RPP) * dv);
  } else {
#pragma unroll
    for (int i = 0; i < RPT; ++i) S[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }

  for (int t = 0; t < T; ++t) {
    const int buf = t & 1;
    const size_t tok = ((size_t)b * T + t) * H + h;
    const size_t tokq = ((size_t)b * T + t) * Hk + hq;
    for (int i = tid; i < DK; i += NT) {
      s_k[buf][i] = to_f32(k[tokq * DK + i]);
      s_q[buf][i] = to_f32(q[tokq * DK + i]);
    }
    const float4 vv = load4(v + tok * dv + col);
    const float alpha = __expf(kGates ? negA * softplus(g[tok] + dtb) : g[tok]);
    const float bt = kGates ? sigmoid(beta[tok]) : beta[tok];
    __syncthreads();

    float4 kh = make_float4(0.f, 0.f, 0.f, 0.f), qh = kh;
    float qk = 0.f;
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const float kr = s_k[buf][rb + i * RPP], qr = s_q[buf][rb + i * RPP];
      kh = fma4(kr, S[i], kh);
      qh = fma4(qr, S[i], qh);
      qk = fmaf(qr, kr, qk);
    }
    // Reduce over the lanes of this warp that hold the same columns.
#pragma unroll
    for (int off = LPR; off < 32; off <<= 1) {
      kh.x += __shfl_xor_sync(0xffffffffu, kh.x, off);
      kh.y += __shfl_xor_sync(0xffffffffu, kh.y, off);
      kh.z += __shfl_xor_sync(0xffffffffu, kh.z, off);
      kh.w += __shfl_xor_sync(0xffffffffu, kh.w, off);
      qh.x += __shfl_xor_sync(0xffffffffu, qh.x, off);
      qh.y += __shfl_xor_sync(0xffffffffu, qh.y, off);
      qh.z += __shfl_xor_sync(0xffffffffu, qh.z, off);
      qh.w += __shfl_xor_sync(0xffffffffu, qh.w, off);
      qk += __shfl_xor_sync(0xffffffffu, qk, off);
    }
    if (lane < LPR) {
      s_red[buf][warp][0][lane] = kh;
      s_red[buf][warp][1][lane] = qh;
      if (lane == 0) s_qk[buf][warp] = qk;
    }
    __syncthreads();
    kh = s_red[buf][0][0][cg];
    qh = s_red[buf][0][1][cg];
    qk = s_qk[buf][0];
#pragma unroll
    for (int w = 1; w < NWARP; ++w) {
      const float4 a = s_red[buf][w][0][cg], c = s_red[buf][w][1][cg];
      kh.x += a.x; kh.y += a.y; kh.z += a.z; kh.w += a.w;
      qh.x += c.x; qh.y += c.y; qh.z += c.z; qh.w += c.w;
      qk += s_qk[buf][w];
    }
    // The lanes summed above hold distinct row groups, so qk now counts every
    // row of q . k exactly once.
    float4 u;
    u.x = bt * (vv.x - alpha * kh.x);
    u.y = bt * (vv.y - alpha * kh.y);
    u.z = bt * (vv.z - alpha * kh.z);
    u.w = bt * (vv.w - alpha * kh.w);
    if (rb == 0) {
      float4 out;
      out.x = fmaf(alpha, qh.x, qk * u.x);
      out.y = fmaf(alpha, qh.y, qk * u.y);
      out.z = fmaf(alpha, qh.z, qk * u.z);
      out.w = fmaf(alpha, qh.w, qk * u.w);
      store4(o + tok * dv + col, out);
    }
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const float kr = s_k[buf][rb + i * RPP];
      S[i] = make_float4(fmaf(alpha, S[i].x, kr * u.x), fmaf(alpha, S[i].y, kr * u.y),
                         fmaf(alpha, S[i].z, kr * u.z), fmaf(alpha, S[i].w, kr * u.w));
    }
  }
  if (hT != nullptr) {
#pragma unroll
    for (int i = 0; i < RPT; ++i) store4_stream(hT + sbase + (size_t)(rb + i * RPP) * dv, S[i]);
  }
}

namespace {

template <typename Tin, int DK, int CW, bool kGates>
cudaError_t launch_cfg(const RecurrentArgs& a, const LayerArgs& la, cudaStream_t st) {
  constexpr int LPR = CW / 4;
  constexpr int NT0 = DK * LPR / 16;  // aim for 16 state rows per thread
  constexpr int NT = NT0 < 32 ? 32 : (NT0 > 256 ? 256 : NT0);
  dim3 grid(a.dv / CW, a.B * a.H);
  recurrent_kernel<Tin, DK, CW, NT, kGates><<<grid, NT, 0, st>>>(
      static_cast<const Tin*>(a.q), static_cast<const Tin*>(a.k), static_cast<const Tin*>(a.v),
      a.g, a.beta, a.h0, static_cast<Tin*>(a.o), a.hT, a.T, a.H, a.Hk, a.dv, la.A_log,
      la.dt_bias);
  return cudaGetLastError();
}

template <typename Tin, int DK, bool kGates>
cudaError_t launch_dk(const RecurrentArgs& a, const LayerArgs& la, cudaStream_t st) {
  if (a.dv % 64 == 0) return launch_cfg<Tin, DK, 64, kGates>(a, la, st);
  if (a.dv % 32 == 0) return launch_cfg<Tin, DK, 32, kGates>(a, la, st);
  return launch_cfg<Tin, DK, 16, kGates>(a, la, st);
}

template <typename Tin, bool kGates>
cudaError_t launch_t(const RecurrentArgs& a, const LayerArgs& la, cudaStream_t st) {
  switch (a.dk) {
    case 16: return launch_dk<Tin, 16, kGates>(a, la, st);
    case 32: return launch_dk<Tin, 32, kGates>(a, la, st);
    case 64: return launch_dk<Tin, 64, kGates>(a, la, st);
    case 128: return launch_dk<Tin, 128, kGates>(a, la, st);
    case 256: return launch_dk<Tin, 256, kGates>(a, la, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_recurrent(const RecurrentArgs& a, cudaStream_t st) {
  if (a.B * a.H == 0 || a.T == 0) return cudaSuccess;
  if (recurrent_bulk_supported(a)) return launch_recurrent_bulk(a, st);
  const LayerArgs none;
  return a.dtype == kBF16 ? launch_t<__nv_bfloat16, false>(a, none, st)
                          : launch_t<float, false>(a, none, st);
}

cudaError_t launch_recurrent_gates(const RecurrentArgs& a, const LayerArgs& la, cudaStream_t st) {
  if (a.B * a.H == 0 || a.T == 0) return cudaSuccess;
  return a.dtype == kBF16 ? launch_t<__nv_bfloat16, true>(a, la, st)
                          : launch_t<float, true>(a, la, st);
}

}  // namespace gdn
