// Chunked gated delta-rule forward on CUDA cores (fp32 arithmetic), sm_100a.
//
// Replaces chunk_gated_delta_rule_fwd (ops.py:299-346).  This is the portable
// path: every supported shape, fp32 or bf16 inputs, both semantics.  The
// tensor-core kernel (chunk_tc.cu) takes the bf16 shapes it is built for.
//
// One CTA owns one (b, h) and a tile of DVT state columns (the dv columns of
// the state evolve independently), and walks the N = ceil(T / C) chunks in
// order.  Per chunk, with in-chunk cumulative gate G, all in shared memory:
//     A   = tril_{-1}(diag(beta) K K^T * e^{G_i - G_j})
//     P   = tril_0(Q K^T * e^{G_i - G_j})
//     X   = diag(beta) (V - diag(e^G) K S)
//     V'  = (I + A)^{-1} X                (forward substitution)
//     O   = diag(e^G) Q S + P V'
//     S  <- e^{G_C} S + (diag(e^{G_C - G}) K)^T V'
// Exponents are formed on the causal triangle only, as e^{G_i - G_j}.
//
// GDN_SEMANTICS_REFERENCE reproduces ops.py as written instead: (I - A)^{-1}
// (ops.py:271-274), the state update with undecayed K (ops.py:329), a decay of
// e^0 after a partial last chunk (the zero re-padding of the cumulated gate,
// ops.py:247/257/327), and the output reshape of ops.py:342 that interleaves
// heads with tokens.
#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {

namespace {

constexpr int kSimtThreads = 256;
constexpr int kMaxChunk = 64;

struct SimtSmem {
  // float offsets into dynamic shared memory
  int K, Q, S, X, QS, A, P, G, eG, dec, bt, total;
};

__host__ __device__ inline SimtSmem simt_layout(int C, int DK, int DVT) {
  SimtSmem L;
  int off = 0;
  L.K = off;  off += C * (DK + 1);
  L.Q = off;  off += C * (DK + 1);
  L.S = off;  off += DK * DVT;
  L.X = off;  off += C * DVT;
  L.QS = off; off += C * DVT;
  L.A = off;  off += C * C;
  L.P = off;  off += C * C;
  L.G = off;  off += C;
  L.eG = off; off += C;
  L.dec = off; off += C;
  L.bt = off; off += C;
  L.total = off;
  return L;
}

// h0 and hT may be the same array (in-place state): each CTA reads its tile of
// h0 before its first chunk and writes the same tile of hT after its last.
template <typename Tin, int DVT>
__global__ void __launch_bounds__(kSimtThreads)
chunk_simt_kernel(const Tin* __restrict__ q, const Tin* __restrict__ k,
                  const Tin* __restrict__ v, const float* __restrict__ g,
                  const float* __restrict__ beta, const float* h0,
                  Tin* __restrict__ o, float* hT,
                  const int* __restrict__ cu_seqlens, int T, int H, int Hk, int DK, int dv,
                  int C, int semantics) {
  constexpr int NT = kSimtThreads;
  constexpr int PARTS = NT / DVT;      // threads sharing one column in the solve
  static_assert(NT % DVT == 0 && PARTS <= 32 && (32 % PARTS) == 0, "solve layout");
  extern __shared__ float smem[];
  const SimtSmem L = simt_layout(C, DK, DVT);
  float* sK = smem + L.K;
  float* sQ = smem + L.Q;
  float* sS = smem + L.S;
  float* sX = smem + L.X;
  float* sQS = smem + L.QS;
  float* sA = smem + L.A;
  float* sP = smem + L.P;
  float* sG = smem + L.G;
  float* seG = smem + L.eG;
  float* sdec = smem + L.dec;
  float* sb = smem + L.bt;
  const int KP = DK + 1;  // padded row stride of K and Q

  const int tid = threadIdx.x;
  const int bh = blockIdx.y;
  int b = bh / H;
  const int h = bh - b * H;
  // Packed variable-length sequences (cu_seqlens != NULL): blockIdx.y = s * H + h,
  // and sequence s is tokens [cu_seqlens[s], cu_seqlens[s + 1]) of the single
  // row of T tokens (offsets clamped to [0, T], so no access leaves the row).
  int tok0 = 0, Tn = T;
  if (cu_seqlens) {
    const int a0 = min(max(cu_seqlens[b], 0), T);
    const int a1 = min(max(cu_seqlens[b + 1], a0), T);
    b = 0, tok0 = a0, Tn = a1 - a0;
  }
  const int c0 = blockIdx.x * DVT;
  const bool literal = semantics == kReference;

  // Initial state tile.
  for (int e = tid; e < DK * DVT; e += NT) {
    const int r = e / DVT, c = e - r * DVT;
    sS[e] = h0 ? h0[((size_t)bh * DK + r) * dv + c0 + c] : 0.f;
  }

  const int N = (Tn + C - 1) / C;
  for (int n = 0; n < N; ++n) {
    const int t0 = n * C;
    __syncthreads();  // previous chunk done with every buffer
    // ---- load the chunk (zero-filled past T) ----
    for (int e = tid; e < C * DK; e += NT) {
      const int i = e / DK, d = e - i * DK;
      const int t = t0 + i;
      float kv = 0.f, qv = 0.f;
      if (t < Tn) {
        // value head h reads q/k head h * Hk / H (grouped heads)
        const size_t off = (((size_t)b * T + tok0 + t) * Hk + h * Hk / H) * DK + d;
        kv = to_f32(k[off]);
        qv = to_f32(q[off]);
      }
      sK[i * KP + d] = kv;
      sQ[i * KP + d] = qv;
    }
    for (int e = tid; e < C * DVT; e += NT) {
      const int i = e / DVT, c = e - i * DVT;
      const int t = t0 + i;
      sX[e] = t < Tn ? to_f32(v[(((size_t)b * T + tok0 + t) * H + h) * dv + c0 + c]) : 0.f;
    }
    if (tid < C) {
      const int t = t0 + tid;
      const size_t off = ((size_t)b * T + tok0 + t) * H + h;
      sG[tid] = t < Tn ? g[off] : 0.f;
      sb[tid] = t < Tn ? beta[off] : 0.f;
    }
    __syncthreads();
    // ---- in-chunk cumulative gate (one warp, serial over <= 64 values) ----
    if (tid == 0) {
      float acc = 0.f;
      for (int i = 0; i < C; ++i) { acc += sG[i]; sG[i] = acc; }
    }
    __syncthreads();
    const float GC = sG[C - 1];
    if (tid < C) {
      seG[tid] = __expf(sG[tid]);
      sdec[tid] = literal ? 1.f : __expf(GC - sG[tid]);
    }
    // ---- A and P (lower triangles) ----
    for (int e = tid; e < C * C; e += NT) {
      const int i = e / C, j = e - i * C;
      float a = 0.f, p = 0.f;
      if (j <= i) {
        float kk = 0.f, qk = 0.f;
        const float* ki = sK + i * KP;
        const float* qi = sQ + i * KP;
        const float* kj = sK + j * KP;
        for (int d = 0; d < DK; ++d) {
          kk = fmaf(ki[d], kj[d], kk);
          qk = fmaf(qi[d], kj[d], qk);
        }
        const float gam = __expf(sG[i] - sG[j]);
        p = qk * gam;
        if (j < i) a = sb[i] * kk * gam;
      }
      sA[e] = a;
      sP[e] = p;
    }
    // ---- K S and Q S; X = beta (V - e^G K S) ----
    __syncthreads();
    for (int e = tid; e < C * DVT; e += NT) {
      const int i = e / DVT, c = e - i * DVT;
      float ks = 0.f, qs = 0.f;
      const float* ki = sK + i * KP;
      const float* qi = sQ + i * KP;
      for (int d = 0; d < DK; ++d) {
        const float s = sS[d * DVT + c];
        ks = fmaf(ki[d], s, ks);
        qs = fmaf(qi[d], s, qs);
      }
      sQS[e] = qs;
      sX[e] = sb[i] * (sX[e] - seG[i] * ks);
    }
    __syncthreads();
    // ---- V' = (I + A)^{-1} X by forward substitution (in place in sX) ----
    {
      const int c = tid / PARTS, part = tid - c * PARTS;
      const float sgn = literal ? 1.f : -1.f;  // (I - A)^{-1} for the literal path
      for (int i = 1; i < C; ++i) {
        float acc = 0.f;
        for (int j = part; j < i; j += PARTS) acc = fmaf(sA[i * C + j], sX[j * DVT + c], acc);
#pragma unroll
        for (int off = 1; off < PARTS; off <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        if (part == 0) sX[i * DVT + c] = fmaf(sgn, acc, sX[i * DVT + c]);
        __syncthreads();
      }
    }
    // ---- O = e^G Q S + P V' ----
    for (int e = tid; e < C * DVT; e += NT) {
      const int i = e / DVT, c = e - i * DVT;
      float acc = seG[i] * sQS[e];
      for (int j = 0; j <= i; ++j) acc = fmaf(sP[i * C + j], sX[j * DVT + c], acc);
      int t = t0 + i, hh = h;
      if (literal) {  // ops.py:342: [N,H,C] order read back as [N*C, H]
        const int f = (n * H + h) * C + i;
        t = f / H;
        hh = f - t * H;
      }
      if (t < Tn) o[(((size_t)b * T + tok0 + t) * H + hh) * dv + c0 + c] = from_f32<Tin>(acc);
    }
    // ---- S <- e^{G_C} S + (e^{G_C - G} K)^T V' ----
    {
      // the literal path decays by e^0 after a zero-padded last chunk
      const float eGC = (literal && t0 + C > Tn) ? 1.f : __expf(GC);
      for (int e = tid; e < DK * DVT; e += NT) {
        const int d = e / DVT, c = e - d * DVT;
        float acc = 0.f;
        for (int i = 0; i < C; ++i) acc = fmaf(sdec[i] * sK[i * KP + d], sX[i * DVT + c], acc);
        sS[e] = fmaf(eGC, sS[e], acc);
      }
    }
  }
  if (hT) {
    __syncthreads();
    for (int e = tid; e < DK * DVT; e += NT) {
      const int r = e / DVT, c = e - r * DVT;
      hT[((size_t)bh * DK + r) * dv + c0 + c] = sS[e];
    }
  }
}

int pick_dvt(const ChunkArgs& a) {
  const int cands[3] = {64, 32, 16};
  for (int dvt : cands) {
    if (a.dv % dvt) continue;
    const size_t bytes = (size_t)simt_layout(a.chunk, a.dk, dvt).total * sizeof(float);
    if (bytes <= 227 * 1024) return dvt;
  }
  return 0;
}

template <typename Tin, int DVT>
cudaError_t launch_simt_t(const ChunkArgs& a, cudaStream_t st) {
  const size_t smem = (size_t)simt_layout(a.chunk, a.dk, DVT).total * sizeof(float);
  auto kern = chunk_simt_kernel<Tin, DVT>;
  static std::atomic<int> smem_set[kMaxDevices] = {};
  cudaError_t e = ensure_smem(kern, (int)smem, smem_set);
  if (e != cudaSuccess) return e;
  dim3 grid(a.dv / DVT, a.B * a.H);
  kern<<<grid, kSimtThreads, smem, st>>>(
      static_cast<const Tin*>(a.q), static_cast<const Tin*>(a.k), static_cast<const Tin*>(a.v),
      a.g, a.beta, a.h0, static_cast<Tin*>(a.o), a.hT, a.cu_seqlens, a.T, a.H, a.Hk, a.dk, a.dv,
      a.chunk,
      a.semantics);
  return cudaGetLastError();
}

template <typename Tin>
cudaError_t launch_simt_dtype(const ChunkArgs& a, cudaStream_t st) {
  switch (pick_dvt(a)) {
    case 64: return launch_simt_t<Tin, 64>(a, st);
    case 32: return launch_simt_t<Tin, 32>(a, st);
    case 16: return launch_simt_t<Tin, 16>(a, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

size_t chunk_simt_smem_bytes(const ChunkArgs& a) {
  if (a.chunk < 1 || a.chunk > kMaxChunk) return 0;
  const int dvt = pick_dvt(a);
  return dvt ? (size_t)simt_layout(a.chunk, a.dk, dvt).total * sizeof(float) : 0;
}

cudaError_t launch_chunk_simt(const ChunkArgs& a, cudaStream_t st) {
  if (a.B * a.H == 0 || a.T == 0) return cudaSuccess;
  return a.dtype == kBF16 ? launch_simt_dtype<__nv_bfloat16>(a, st)
                          : launch_simt_dtype<float>(a, st);
}

}  // namespace gdn
