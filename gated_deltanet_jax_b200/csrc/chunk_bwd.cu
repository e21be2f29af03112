// Backward of the chunked gated delta rule (exact semantics) on the tensor cores.
//
// The reference has no backward of its own: it relies on JAX autodiff of its
// chunk path (ops.py:238-346).  This computes the gradients of the recurrence
// (ops.py:170-184 with an initial / final state) by reverse-mode
// differentiation through its chunked form, term for term the oracle's
// chunk_exact_backward, rearranged so that only two or three short products
// per chunk are sequential.
//
// Per chunk of C tokens (in-chunk cumulative gate G, gamma = G_C, e = e^G,
// d = e^{gamma - G}), with T = (I + A)^{-1}, A = tril_{-1}(beta_i K_i.K_j e^{G_i-G_j}),
// P = tril_0(Q_i.K_j e^{G_i-G_j}) and the state h entering the chunk:
//
//   forward   V' = U - W h,          h_out = e^gamma h + K^T (d V')
//             W = T diag(beta e) K,   U = T diag(beta) V
//   backward  dX = Y + Z dh_out,      dh = e^gamma dh_out + Q^T (e dO) - K^T (beta e dX)
//             Y = T^T P^T dO,         Z = T^T diag(d) K
//   (dX = T^T dV' is the gradient of X = diag(beta)(V - diag(e) K h), with
//    dV' = P^T dO + diag(d) K dh_out.)
//
// and, per chunk once h, dh_out, V' and dX are known,
//
//   dA = -tril_{-1}(dX V'^T), dP = tril_0(dO V'^T), dPE = dP e^{G_i-G_j}, dAE = dA e^{G_i-G_j}
//   dQ = e (dO h^T) + dPE K
//   dK = d (V' dh_out^T) - beta e (dX h^T) + dPE^T Q + beta (dAE K) + dAE^T (beta K)
//   dV = beta dX
//   dbeta = rowsum(dX o V) - e rowsum(K o dX h^T) + rowsum(dAE o K K^T)
//   dG = -d rowsum(K o V' dh_out^T) + e rowsum(Q o dO h^T) - beta e rowsum(K o dX h^T)
//        + rowsum - colsum of (dPE o Q K^T) and of (dAE o beta K K^T)
//   dG_C += e^gamma <h, dh_out> + sum(d K o V' dh_out^T);  dg = reverse in-chunk cumsum of dG.
//
// Launches, in order on the caller's stream:
//   1. bwd_prep    one CTA per (chunk, value head): T, W, U, Y, Z.
//   2. bwd_states  one CTA per (32-column state tile, value head, direction):
//                  the forward pass stores every chunk's entering state and V';
//                  the reverse pass stores every chunk's dh_out and dX, and dh0.
//   3. bwd_grads   one CTA per (chunk, value head): every gradient of the chunk.
//   4. bwd_group   (grouped q/k heads only) sums dq, dk over each head group.
// Every product runs on the tensor cores (warp-level mma.sync, tf32 operands,
// fp32 accumulation; three-term tf32 splitting for fp32 inputs) from fp32
// tiles in shared memory.  Nothing is summed with atomics, so the gradients
// are the same on every run.
#include <cstdint>

#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {

namespace {

constexpr int C = 64;        // chunk length (the exact result does not depend on it)
constexpr int NT = 256;      // threads per CTA (8 warps)
constexpr int KT = 32;       // dk columns per streamed tile
constexpr int VT = 32;       // dv columns per streamed tile and per state tile
// Shared-memory row strides.  A fragment load reads 8 rows x 4 columns
// (row stride = 4 banks apart: conflict-free) or 4 rows x 8 columns (8 banks
// apart: conflict-free); the other pattern on the same matrix is 2-way.
constexpr int LC = C + 4;    // C x C matrices
constexpr int LT = VT + 4;   // 32-column tiles read by rows
constexpr int LB = VT + 8;   // 32-column tiles read by columns

struct BwdParams {
  const void* q; const void* k; const void* v; const void* dO;
  const float* g; const float* beta; const float* h0; const float* dhT;
  void* dq; void* dk_out; void* dv_out; float* dg; float* dbeta; float* dh0;
  // workspace
  float* W;     // [B*H][Np][ldw]     ldw = dk rounded up to 32, zero past dk
  float* Z;     // [B*H][Np][ldw]
  float* UV;    // [B*H][Np][dv]      U, then V'
  float* YX;    // [B*H][Np][dv]      Y, then dX
  float* hs;    // [B*H][N][dk][dv]   state entering chunk n
  float* dhs;   // [B*H][N][dk][dv]   gradient of the state leaving chunk n
  float* dqk;   // [2][tokens][H][dk] per value head dq, dk (grouped heads only)
  // Sequences: dense, B sequences of T tokens ([B, T, ...] is one row of B T
  // tokens), N chunks each; packed (cu != NULL), n_seqs sequences of one row
  // of T tokens, sequence s the tokens [cu[s], cu[s + 1]) and its chunks
  // coff[s] .. coff[s + 1] - 1.  Chunk c of every head owns workspace rows
  // (c H + h) C .. + C - 1 and state tile c H + h.
  const int* cu;
  const int* coff;
  int n_seqs;
  int B, T, H, Hk, dk, dv, N, ldw;
  // The forward on these kernels (dO == NULL): the final state (or NULL) and o.
  float* hTout = nullptr;
  void* o = nullptr;
  // The state kernel's reverse direction only (the forward pass ran elsewhere).
  int rev_only = 0;
};

// Tokens and chunks of sequence s.
struct SeqSpan {
  size_t tok0;   // first token in the packed row
  int len;       // tokens
  int cfirst;    // first global chunk
  int nch;       // chunks
};

__device__ __forceinline__ SeqSpan seq_span(const BwdParams& p, int s) {
  SeqSpan r;
  if (!p.cu) {
    r.tok0 = (size_t)s * p.T; r.len = p.T; r.cfirst = s * p.N; r.nch = p.N;
  } else {
    const int a0 = min(max(p.cu[s], 0), p.T);
    const int a1 = min(max(p.cu[s + 1], a0), p.T);
    r.tok0 = (size_t)a0; r.len = a1 - a0; r.cfirst = p.coff[s]; r.nch = p.coff[s + 1] - p.coff[s];
  }
  return r;
}

// The sequence that global chunk c belongs to, or -1 past the last chunk.
__device__ __forceinline__ int seq_of_chunk(const BwdParams& p, int c) {
  if (!p.cu) return c < p.B * p.N ? c / p.N : -1;
  if (c >= p.coff[p.n_seqs]) return -1;
  int lo = 0, hi = p.n_seqs;   // coff[lo] <= c < coff[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (p.coff[mid] <= c) lo = mid; else hi = mid;
  }
  return lo;
}

// ---------------------------------------------------------------------------
// Warp-level tensor-core products: mma.sync m16n8k8 with tf32 operands and
// fp32 accumulators.  bf16 inputs are exact in tf32, fp32 intermediates are
// rounded to tf32 (11 significant bits).  With kSplit (fp32 inputs) every
// operand is split as x = hi + lo (both tf32) and a b ~ hi_a hi_b + hi_a lo_b
// + lo_a hi_b, which keeps about fp32 accuracy.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4],
                                         const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

template <bool kSplit>
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
  hi = to_tf32(x);
  if (kSplit) lo = to_tf32(x - __uint_as_float(hi));
}

// acc[i][j] += sum_{k < K} a(m, k) b(k, n) over the warp's MT x NTL tiles of
// 16 x 8 at (m0 + 16 i, n0 + 8 j), with a(m, k) = TA ? A[k lda + m] : A[m lda + k]
// and b(k, n) = TB ? B[n ldb + k] : B[k ldb + n].  K is a multiple of 8.
// Accumulator element e of tile (i, j) is row m0 + 16 i + g + 8 (e >> 1),
// column n0 + 8 j + 2 t + (e & 1), for lane = 4 g + t.
template <int MT, int NTL, bool TA, bool TB, bool kSplit>
__device__ __forceinline__ void warp_mma(float (&acc)[MT][NTL][4], const float* A, int lda,
                                         const float* B, int ldb, int m0, int n0, int K) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll 2
  for (int k0 = 0; k0 < K; k0 += 8) {
    uint32_t ah[MT][4], al[MT][4], bh[NTL][2], bl[NTL][2];
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int m = m0 + 16 * i + g + 8 * (e & 1), kk = k0 + t + 4 * (e >> 1);
        split_tf32<kSplit>(TA ? A[kk * lda + m] : A[m * lda + kk], ah[i][e], al[i][e]);
      }
#pragma unroll
    for (int j = 0; j < NTL; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int n = n0 + 8 * j + g, kk = k0 + t + 4 * e;
        split_tf32<kSplit>(TB ? B[n * ldb + kk] : B[kk * ldb + n], bh[j][e], bl[j][e]);
      }
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
      for (int j = 0; j < NTL; ++j) {
        mma_tf32(acc[i][j], ah[i], bh[j]);
        if (kSplit) {
          mma_tf32(acc[i][j], ah[i], bl[j]);
          mma_tf32(acc[i][j], al[i], bh[j]);
        }
      }
  }
}

template <int MT, int NTL>
__device__ __forceinline__ void zero(float (&acc)[MT][NTL][4]) {
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < NTL; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.f;
}

// Row and column of accumulator element e of tile (i, j) (see warp_mma).
struct Frag {
  int g, t;
  __device__ Frag() : g((threadIdx.x & 31) >> 2), t(threadIdx.x & 3) {}
  __device__ int row(int m0, int i, int e) const { return m0 + 16 * i + g + 8 * (e >> 1); }
  __device__ int col(int n0, int j, int e) const { return n0 + 8 * j + 2 * t + (e & 1); }
};

// Sum over the 4 lanes of a quad (the lanes holding one accumulator row).
__device__ __forceinline__ float quad_sum(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  return x + __shfl_xor_sync(0xffffffffu, x, 2);
}
// Sum over the 8 quads (the lanes holding one accumulator column).
__device__ __forceinline__ float column_sum(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 4);
  x += __shfl_xor_sync(0xffffffffu, x, 8);
  return x + __shfl_xor_sync(0xffffffffu, x, 16);
}

// Two adjacent output elements (col even) in the output dtype.
__device__ __forceinline__ void store2(float* p, float a, float b) {
  *reinterpret_cast<float2*>(p) = make_float2(a, b);
}
__device__ __forceinline__ void store2(__nv_bfloat16* p, float a, float b) {
  *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
}

// Four or eight input elements (16 bytes) as fp32.
template <typename Tin> __device__ __forceinline__ void unpack16(const uint4& u, float* f);
template <> __device__ __forceinline__ void unpack16<float>(const uint4& u, float* f) {
  f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
  f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
}
template <> __device__ __forceinline__ void unpack16<__nv_bfloat16>(const uint4& u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// VE consecutive floats into shared memory at dst (16-byte stores when the
// row stride LD keeps them aligned).
template <int LD, int VE>
__device__ __forceinline__ void put_row(float* dst, const float* f, float sc) {
  if constexpr (LD % 4 == 0) {
#pragma unroll
    for (int j = 0; j < VE; j += 4)
      *reinterpret_cast<float4*>(dst + j) =
          make_float4(f[j] * sc, f[j + 1] * sc, f[j + 2] * sc, f[j + 3] * sc);
  } else {
#pragma unroll
    for (int j = 0; j < VE; ++j) dst[j] = f[j] * sc;
  }
}

// A C x W tile of one head of a [rows, heads, D] input: rows t0 .. t0+C-1 of
// the sequence starting at row bT, columns c0 .. c0+W-1, zero past the
// sequence's end (T) and past D.  fetch() issues the thread's 16-byte loads
// into registers (inputs are 16-byte aligned, D a multiple of 8 elements);
// put() converts them to fp32 and stores them into shared memory (row stride
// LD), times rowscale[r] if given.  Between the two the loads are in flight,
// so a tile fetched before a product arrives while the product runs.
template <int W, typename Tin>
struct TokenTile {
  static constexpr int VE = 16 / (int)sizeof(Tin), PR = W / VE, NV = C * PR / NT;
  static_assert(W % VE == 0 && (C * PR) % NT == 0, "tile must split evenly into vectors");
  uint4 raw[NV];

  __device__ __forceinline__ void fetch(const Tin* src, size_t bT, int t0, int T, int heads,
                                        int hd, int D, int c0) {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int e = threadIdx.x + i * NT, r = e / PR, col = c0 + (e - r * PR) * VE, t = t0 + r;
      raw[i] = make_uint4(0u, 0u, 0u, 0u);
      if (t < T && col < D)
        raw[i] = __ldg(reinterpret_cast<const uint4*>(src + ((bT + t) * heads + hd) * D + col));
    }
  }
  template <int LD>
  __device__ __forceinline__ void put(float* s, const float* rowscale) const {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int e = threadIdx.x + i * NT, r = e / PR, cv = (e - r * PR) * VE;
      float f[VE];
      unpack16<Tin>(raw[i], f);
      put_row<LD, VE>(s + r * LD + cv, f, rowscale ? rowscale[r] : 1.f);
    }
  }
};

// C rows x W columns (from c0) of a row-major [rows][D] fp32 workspace block
// (D a multiple of 4, 16-byte aligned rows), zero past D; fetch / put as
// TokenTile.
template <int W>
struct BlockTile {
  static constexpr int PR = W / 4, NV = C * PR / NT;
  static_assert((C * PR) % NT == 0, "tile must split evenly into vectors");
  float4 raw[NV];

  __device__ __forceinline__ void fetch(const float* src, int D, int c0) {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int e = threadIdx.x + i * NT, r = e / PR, col = c0 + (e - r * PR) * 4;
      raw[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (col < D) raw[i] = *reinterpret_cast<const float4*>(src + (size_t)r * D + col);
    }
  }
  template <int LD>
  __device__ __forceinline__ void put(float* s) const {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int e = threadIdx.x + i * NT, r = e / PR, cv = (e - r * PR) * 4;
      const float f[4] = {raw[i].x, raw[i].y, raw[i].z, raw[i].w};
      put_row<LD, 4>(s + r * LD + cv, f, 1.f);
    }
  }
};

template <int W, int LD, typename Tin>
__device__ __forceinline__ void load_tokens(float* s, const Tin* src, size_t bT, int t0, int T,
                                            int heads, int hd, int D, int c0,
                                            const float* rowscale) {
  TokenTile<W, Tin> tile;
  tile.fetch(src, bT, t0, T, heads, hd, D, c0);
  tile.template put<LD>(s, rowscale);
}

template <int W, int LD>
__device__ __forceinline__ void load_block(float* s, const float* src, int D, int c0) {
  BlockTile<W> tile;
  tile.fetch(src, D, c0);
  tile.template put<LD>(s);
}

// Gate vectors of one chunk (warp 0): G (inclusive cumulative gate), e^G,
// e^{gamma - G}, beta, beta e^G.  Tokens past the sequence's end have g = beta = 0.
struct GateRegs {
  float x0, x1, b0, b1;   // g and beta of tokens lane and lane + 32 (warp 0)
};

__device__ __forceinline__ void gates_fetch(GateRegs& r, const BwdParams& p, size_t base, int Tn,
                                            int h, int t0) {
  if (threadIdx.x >= 32) return;
  const int l = threadIdx.x;
  const int ta = t0 + l, tb = t0 + 32 + l;
  r.x0 = ta < Tn ? p.g[(base + ta) * p.H + h] : 0.f;
  r.x1 = tb < Tn ? p.g[(base + tb) * p.H + h] : 0.f;
  r.b0 = ta < Tn ? p.beta[(base + ta) * p.H + h] : 0.f;
  r.b1 = tb < Tn ? p.beta[(base + tb) * p.H + h] : 0.f;
}

__device__ __forceinline__ void gates_put(const GateRegs& r, float* sG, float* se, float* sd,
                                          float* sb, float* sbe) {
  if (threadIdx.x >= 32) return;
  const int l = threadIdx.x;
  float x0 = r.x0, x1 = r.x1;
  const float b0 = r.b0, b1 = r.b1;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y0 = __shfl_up_sync(0xffffffffu, x0, o);
    const float y1 = __shfl_up_sync(0xffffffffu, x1, o);
    if (l >= o) { x0 += y0; x1 += y1; }
  }
  x1 += __shfl_sync(0xffffffffu, x0, 31);
  const float gam = __shfl_sync(0xffffffffu, x1, 31);
  sG[l] = x0; sG[l + 32] = x1;
  const float e0 = gate_exp(x0), e1 = gate_exp(x1);
  se[l] = e0; se[l + 32] = e1;
  sd[l] = gate_exp(gam - x0); sd[l + 32] = gate_exp(gam - x1);
  sb[l] = b0; sb[l + 32] = b1;
  sbe[l] = b0 * e0; sbe[l + 32] = b1 * e1;
}

__device__ __forceinline__ void chunk_gates(const BwdParams& p, size_t base, int Tn, int h, int t0,
                                            float* sG, float* se, float* sd, float* sb,
                                            float* sbe) {
  GateRegs r;
  gates_fetch(r, p, base, Tn, h, t0);
  gates_put(r, sG, se, sd, sb, sbe);
}

// ---------------------------------------------------------------------------
// 1. per chunk: T, W, U, Y, Z
// ---------------------------------------------------------------------------
constexpr int kPrepSmemFloats = 3 * C * LC + 3 * C * LB + 5 * C;

template <typename Tin>
__global__ void __launch_bounds__(NT, 2) bwd_prep_kernel(const BwdParams p) {
  constexpr bool kSplit = sizeof(Tin) == 4;
  extern __shared__ float sm[];
  float* sA = sm;
  float* sT = sA + C * LC;
  float* sP = sT + C * LC;
  float* s1 = sP + C * LC;          // C x 32 tiles (stride LT for Q K^T, LB after)
  float* s2 = s1 + C * LB;
  float* s3 = s2 + C * LB;
  float* sG = s3 + C * LB;
  float* se = sG + C; float* sd = se + C; float* sb = sd + C; float* sbe = sb + C;
  const Tin* q = static_cast<const Tin*>(p.q);
  const Tin* k = static_cast<const Tin*>(p.k);
  const Tin* v = static_cast<const Tin*>(p.v);
  const Tin* dO = static_cast<const Tin*>(p.dO);
  const int gc = blockIdx.x, h = blockIdx.y, sq = seq_of_chunk(p, gc);
  if (sq < 0) return;   // past the last chunk (packed sequences)
  const SeqSpan sp = seq_span(p, sq);
  const int n = gc - sp.cfirst, Tn = sp.len;
  const int hq = h * p.Hk / p.H, t0 = n * C, tid = threadIdx.x, w = tid >> 5;
  const size_t bT = sp.tok0;
  const size_t row0 = ((size_t)gc * p.H + h) * C;
  const Frag f;
  chunk_gates(p, bT, Tn, h, t0, sG, se, sd, sb, sbe);

  // Q K^T and K K^T over dk tiles; warp: rows mq.., columns nq..
  const int mq = (w >> 1) * 16, nq = (w & 1) * 32;
  float aQK[1][4][4], aKK[1][4][4];
  zero(aQK); zero(aKK);
  // every tile loop below fetches its next tile before the current products
  TokenTile<KT, Tin> t1, t2;
  t1.fetch(q, bT, t0, Tn, p.Hk, hq, p.dk, 0);
  t2.fetch(k, bT, t0, Tn, p.Hk, hq, p.dk, 0);
  for (int c0 = 0; c0 < p.dk; c0 += KT) {
    __syncthreads();
    t1.put<LT>(s1, nullptr);
    t2.put<LT>(s2, nullptr);
    __syncthreads();
    if (c0 + KT < p.dk) {
      t1.fetch(q, bT, t0, Tn, p.Hk, hq, p.dk, c0 + KT);
      t2.fetch(k, bT, t0, Tn, p.Hk, hq, p.dk, c0 + KT);
    }
    warp_mma<1, 4, false, true, kSplit>(aQK, s1, LT, s2, LT, mq, nq, KT);
    warp_mma<1, 4, false, true, kSplit>(aKK, s2, LT, s2, LT, mq, nq, KT);
  }
  t2.fetch(k, bT, t0, Tn, p.Hk, hq, p.dk, 0);   // first K tile of W, Z (arrives during T)
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int m = f.row(mq, 0, e), c = f.col(nq, j, e);
      const float E = c <= m ? gate_exp(sG[m] - sG[c]) : 0.f;
      sA[m * LC + c] = c < m ? sb[m] * aKK[0][j][e] * E : 0.f;
      sP[m * LC + c] = aQK[0][j][e] * E;
    }
  __syncthreads();
  // T = (I + A)^{-1} by forward substitution: column c by the lane quad g of
  // warp c / 8, one row after another (each lane sums every fourth term)
  {
    const int c = w * 8 + f.g;
    for (int r = 0; r < C; ++r) {
      float s = 0.f;
      for (int j = c + f.t; j < r; j += 4) s = fmaf(sA[r * LC + j], sT[j * LC + c], s);
      s = quad_sum(s);
      if (f.t == 0) sT[r * LC + c] = r < c ? 0.f : (r == c ? 1.f : -s);
      __syncwarp();
    }
  }
  // W = T (beta e K), Z = T^T (d K) per dk tile (columns past dk are zero)
  const int mw = (w >> 1) * 16, nw = (w & 1) * 16;
  for (int c0 = 0; c0 < p.ldw; c0 += KT) {
    __syncthreads();
    t2.put<LB>(s1, sbe);
    t2.put<LB>(s2, sd);
    __syncthreads();
    if (c0 + KT < p.ldw) {
      t2.fetch(k, bT, t0, Tn, p.Hk, hq, p.dk, c0 + KT);
    } else {   // first tiles of U, Y
      t1.fetch(v, bT, t0, Tn, p.H, h, p.dv, 0);
      if (dO) t2.fetch(dO, bT, t0, Tn, p.H, h, p.dv, 0);
    }
    float aw[1][2][4], az[1][2][4];
    zero(aw); zero(az);
    warp_mma<1, 2, false, false, kSplit>(aw, sT, LC, s1, LB, mw, nw, C);
    if (dO) warp_mma<1, 2, true, false, kSplit>(az, sT, LC, s2, LB, mw, nw, C);
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const size_t off = (row0 + f.row(mw, 0, e)) * p.ldw + c0 + f.col(nw, j, e);
        store2(p.W + off, aw[0][j][e], aw[0][j][e + 1]);
        if (dO) store2(p.Z + off, az[0][j][e], az[0][j][e + 1]);
      }
  }
  // U = T (beta V), Y = T^T (P^T dO) per dv tile (the forward: U only)
  for (int c0 = 0; c0 < p.dv; c0 += VT) {
    __syncthreads();
    t1.put<LB>(s1, sb);
    if (dO) t2.put<LB>(s2, nullptr);
    __syncthreads();
    if (c0 + VT < p.dv) {
      t1.fetch(v, bT, t0, Tn, p.H, h, p.dv, c0 + VT);
      if (dO) t2.fetch(dO, bT, t0, Tn, p.H, h, p.dv, c0 + VT);
    }
    float au[1][2][4], ap[1][2][4];
    zero(au); zero(ap);
    warp_mma<1, 2, false, false, kSplit>(au, sT, LC, s1, LB, mw, nw, C);
    if (dO) warp_mma<1, 2, true, false, kSplit>(ap, sP, LC, s2, LB, mw, nw, C);
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const int m = f.row(mw, 0, e), c = f.col(nw, j, e);
        store2(p.UV + (row0 + m) * p.dv + c0 + c, au[0][j][e], au[0][j][e + 1]);
        if (dO) store2(s3 + m * LB + c, ap[0][j][e], ap[0][j][e + 1]);
      }
    if (!dO) continue;
    __syncthreads();
    float ay[1][2][4];
    zero(ay);
    warp_mma<1, 2, true, false, kSplit>(ay, sT, LC, s3, LB, mw, nw, C);
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const int m = f.row(mw, 0, e), c = f.col(nw, j, e);
        store2(p.YX + (row0 + m) * p.dv + c0 + c, ay[0][j][e], ay[0][j][e + 1]);
      }
  }
}

// ---------------------------------------------------------------------------
// 2. the two sequential passes over the chunks
// ---------------------------------------------------------------------------
// Warp tiles of the DKP x VT state product.
template <int DKP> struct StateTiles;
template <> struct StateTiles<256> {
  static constexpr int MT = 4, NTL = 2;
  static __device__ int m0(int w) { return (w >> 1) * 64; }
  static __device__ int n0(int w) { return (w & 1) * 16; }
};
template <> struct StateTiles<128> {
  static constexpr int MT = 2, NTL = 2;
  static __device__ int m0(int w) { return (w >> 1) * 32; }
  static __device__ int n0(int w) { return (w & 1) * 16; }
};
template <> struct StateTiles<64> {
  static constexpr int MT = 1, NTL = 2;
  static __device__ int m0(int w) { return (w >> 1) * 16; }
  static __device__ int n0(int w) { return (w & 1) * 16; }
};
template <> struct StateTiles<32> {
  static constexpr int MT = 1, NTL = 1;
  static __device__ int m0(int w) { return (w >> 2) * 16; }
  static __device__ int n0(int w) { return (w & 3) * 8; }
};

constexpr int SS = VT + 8;   // state tile row stride (read by columns)

template <int DKP>
constexpr int states_smem_floats() {
  return DKP * SS + C * (DKP + 4) + C * (DKP + 8) + 2 * C * LB + 5 * C;
}

// (DKP = 256: 197 KB of shared memory, one CTA per SM, and the registers for
// its 256-column prefetch tiles)
template <typename Tin, int DKP>
__global__ void __launch_bounds__(NT, DKP == 256 ? 1 : 2) bwd_states_kernel(const BwdParams p) {
  using ST = StateTiles<DKP>;
  constexpr bool kSplit = sizeof(Tin) == 4;
  constexpr int LW = DKP + 4, LK = DKP + 8;
  extern __shared__ float sm[];
  float* sS = sm;                   // DKP x SS  state (or state gradient) tile
  float* sM = sS + DKP * SS;        // C x LW    W | Z, then Q
  float* sK = sM + C * LW;          // C x LK    K
  float* sU = sK + C * LK;          // C x LB    U -> d V'  |  Y -> -beta e dX
  float* sO = sU + C * LB;          // C x LB    e dO
  float* sG = sO + C * LB;
  float* se = sG + C; float* sd = se + C; float* sb = sd + C; float* sbe = sb + C;
  const Tin* q = static_cast<const Tin*>(p.q);
  const Tin* k = static_cast<const Tin*>(p.k);
  const Tin* dO = static_cast<const Tin*>(p.dO);
  const int c0 = blockIdx.x * VT, bh = blockIdx.y, sq = bh / p.H, h = bh - sq * p.H;
  const int hq = h * p.Hk / p.H, tid = threadIdx.x, w = tid >> 5;
  const bool rev = blockIdx.z != 0 || p.rev_only;
  const SeqSpan sp = seq_span(p, sq);
  const size_t bT = sp.tok0;
  const int Tn = sp.len;
  const Frag f;
  const int mv = (w >> 1) * 16, nv = (w & 1) * 16;       // C x VT products
  const int ms = ST::m0(w), ns = ST::n0(w);              // DKP x VT products
  const float* init = rev ? p.dhT : p.h0;
  for (int e = tid; e < DKP * VT; e += NT) {
    const int r = e / VT, c = e - r * VT;
    sS[r * SS + c] = (init && r < p.dk) ? init[((size_t)bh * p.dk + r) * p.dv + c0 + c] : 0.f;
  }
  float* keep = rev ? p.dhs : p.hs;
  for (int it = 0; it < sp.nch; ++it) {
    const int n = rev ? sp.nch - 1 - it : it, t0 = n * C, gc = sp.cfirst + n;
    const size_t row0 = ((size_t)gc * p.H + h) * C;
    // every global load of the step is issued here, before the first wait (fp32
    // inputs: the reverse pass's Q, K, dO after the dX product -- their rows
    // would need twice the registers)
    constexpr bool kEarly = sizeof(Tin) == 2;
    BlockTile<DKP> tM;
    BlockTile<VT> tU;
    TokenTile<DKP, Tin> tK, tQ;
    TokenTile<VT, Tin> tO;
    GateRegs gr;
    tM.fetch((rev ? p.Z : p.W) + row0 * p.ldw, p.ldw, 0);
    tU.fetch((rev ? p.YX : p.UV) + row0 * p.dv, p.dv, c0);
    gates_fetch(gr, p, bT, Tn, h, t0);
    if (!rev || kEarly) tK.fetch(k, bT, t0, Tn, p.Hk, hq, p.dk, 0);
    if (rev && kEarly) {
      tQ.fetch(q, bT, t0, Tn, p.Hk, hq, p.dk, 0);
      tO.fetch(dO, bT, t0, Tn, p.H, h, p.dv, c0);
    }
    __syncthreads();
    for (int e = tid * 4; e < DKP * VT; e += NT * 4) {
      const int r = e / VT, c = e - r * VT;
      if (r < p.dk)
        *reinterpret_cast<float4*>(keep + (((size_t)gc * p.H + h) * p.dk + r) * p.dv + c0 + c) =
            *reinterpret_cast<const float4*>(sS + r * SS + c);
    }
    tM.put<LW>(sM);
    tU.put<LB>(sU);
    gates_put(gr, sG, se, sd, sb, sbe);
    if (!rev) tK.put<LK>(sK, nullptr);
    __syncthreads();
    // forward: V' = U - W h;  reverse: dX = Y + Z dh
    float acc[1][2][4];
    zero(acc);
    warp_mma<1, 2, false, false, kSplit>(acc, sM, LW, sS, SS, mv, nv, DKP);
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const int m = f.row(mv, 0, e), c = f.col(nv, j, e);
        float* u = sU + m * LB + c;
        const size_t off = (row0 + m) * p.dv + c0 + c;
        if (!rev) {
          const float v0 = u[0] - acc[0][j][e], v1 = u[1] - acc[0][j][e + 1];
          store2(p.UV + off, v0, v1);
          u[0] = sd[m] * v0; u[1] = sd[m] * v1;
        } else {
          const float x0 = u[0] + acc[0][j][e], x1 = u[1] + acc[0][j][e + 1];
          store2(p.YX + off, x0, x1);
          u[0] = -sbe[m] * x0; u[1] = -sbe[m] * x1;
        }
      }
    if (rev) {
      if (!kEarly) {
        tK.fetch(k, bT, t0, Tn, p.Hk, hq, p.dk, 0);
        tQ.fetch(q, bT, t0, Tn, p.Hk, hq, p.dk, 0);
        tO.fetch(dO, bT, t0, Tn, p.H, h, p.dv, c0);
      }
      __syncthreads();   // Z in sM has been read; sM now takes Q
      tQ.put<LW>(sM, nullptr);
      tK.put<LK>(sK, nullptr);
      tO.put<LB>(sO, se);
    }
    __syncthreads();
    // forward: h = e^gamma h + K^T (d V');  reverse: dh = e^gamma dh + Q^T (e dO) + K^T (-beta e dX)
    float accS[ST::MT][ST::NTL][4];
    zero(accS);
    warp_mma<ST::MT, ST::NTL, true, false, kSplit>(accS, sK, LK, sU, LB, ms, ns, C);
    if (rev) warp_mma<ST::MT, ST::NTL, true, false, kSplit>(accS, sM, LW, sO, LB, ms, ns, C);
    const float eg = se[C - 1];
#pragma unroll
    for (int i = 0; i < ST::MT; ++i)
#pragma unroll
      for (int j = 0; j < ST::NTL; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float* s = sS + f.row(ms, i, e) * SS + f.col(ns, j, e);
          *s = fmaf(eg, *s, accS[i][j][e]);
        }
  }
  if (rev && p.dh0) {
    __syncthreads();
    for (int e = tid; e < DKP * VT; e += NT) {
      const int r = e / VT, c = e - r * VT;
      if (r < p.dk) p.dh0[((size_t)bh * p.dk + r) * p.dv + c0 + c] = sS[r * SS + c];
    }
  }
  if (!rev && p.hTout) {   // the forward on these kernels: the final state
    __syncthreads();
    for (int e = tid; e < DKP * VT; e += NT) {
      const int r = e / VT, c = e - r * VT;
      if (r < p.dk) p.hTout[((size_t)bh * p.dk + r) * p.dv + c0 + c] = sS[r * SS + c];
    }
  }
}

// ---------------------------------------------------------------------------
// The forward on these kernels, for the shapes the tcgen05 kernel does not take
// (fp32 inputs; bf16 with dk < 128 or dv not a multiple of 64): bwd_prep
// without dO (T, W, U), the forward state pass (V' = U - W h and every chunk's
// entering state h, the final state), then per chunk
//   O = e^G (Q h) + P V',   P = tril_0(Q K^T e^{G_i - G_j})
// on the same warp-level products (three-term tf32 for fp32 inputs).
// ---------------------------------------------------------------------------
template <int DKP>
constexpr int out_smem_floats() {
  return C * (DKP + 4) + C * LT + C * LC + KT * LB + C * LB + 5 * C;
}

template <typename Tin, int DKP>
__global__ void __launch_bounds__(NT, 2) fwd_out_kernel(const BwdParams p) {
  constexpr bool kSplit = sizeof(Tin) == 4;
  constexpr int LQ = DKP + 4;
  extern __shared__ float sm[];
  float* sQ = sm;                 // C x LQ   Q, every key column (zero past dk)
  float* sK = sQ + C * LQ;        // C x LT   one 32-column tile of K
  float* sP = sK + C * LT;        // C x LC   P
  float* sH = sP + C * LC;        // KT x LB  32 x 32 tile of the entering state
  float* sV = sH + KT * LB;       // C x LB   32-column tile of V'
  float* sG = sV + C * LB;
  float* se = sG + C; float* sd = se + C; float* sb = sd + C; float* sbe = sb + C;
  const Tin* q = static_cast<const Tin*>(p.q);
  const Tin* k = static_cast<const Tin*>(p.k);
  Tin* o = static_cast<Tin*>(p.o);
  const int gc = blockIdx.x, h = blockIdx.y, sq = seq_of_chunk(p, gc);
  if (sq < 0) return;
  const SeqSpan sp = seq_span(p, sq);
  const int n = gc - sp.cfirst, Tn = sp.len;
  const int hq = h * p.Hk / p.H, t0 = n * C, tid = threadIdx.x, w = tid >> 5;
  const size_t bT = sp.tok0;
  const size_t row0 = ((size_t)gc * p.H + h) * C;
  const Frag f;
  chunk_gates(p, bT, Tn, h, t0, sG, se, sd, sb, sbe);
  {
    TokenTile<DKP, Tin> tQ;
    tQ.fetch(q, bT, t0, Tn, p.Hk, hq, p.dk, 0);
    tQ.put<LQ>(sQ, nullptr);
  }
  // P = tril_0(Q K^T e^{G_i - G_j}); warp: rows mq.., columns nq..
  const int mq = (w >> 1) * 16, nq = (w & 1) * 32;
  float aQK[1][4][4];
  zero(aQK);
  TokenTile<KT, Tin> tK;
  tK.fetch(k, bT, t0, Tn, p.Hk, hq, p.dk, 0);
  for (int c0 = 0; c0 < p.dk; c0 += KT) {
    __syncthreads();
    tK.put<LT>(sK, nullptr);
    __syncthreads();
    if (c0 + KT < p.dk) tK.fetch(k, bT, t0, Tn, p.Hk, hq, p.dk, c0 + KT);
    warp_mma<1, 4, false, true, kSplit>(aQK, sQ + c0, LQ, sK, LT, mq, nq, KT);
  }
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int m = f.row(mq, 0, e), c = f.col(nq, j, e);
      sP[m * LC + c] = c <= m ? aQK[0][j][e] * gate_exp(sG[m] - sG[c]) : 0.f;
    }
  // O, 32 columns at a time: e^G (Q h) over 32-row tiles of h, then + P V'
  const int mv = (w >> 1) * 16, nv = (w & 1) * 16;
  const float* hs = p.hs + ((size_t)gc * p.H + h) * p.dk * p.dv;
  for (int c0 = 0; c0 < p.dv; c0 += VT) {
    BlockTile<VT> tU;
    tU.fetch(p.UV + row0 * p.dv, p.dv, c0);
    float acc[1][2][4];
    zero(acc);
    for (int kt = 0; kt < p.dk; kt += KT) {
      __syncthreads();   // the previous tiles' readers are done (first pass: P is written)
      for (int e = tid * 4; e < KT * VT; e += NT * 4) {
        const int r = e / VT, c = e - r * VT;
        *reinterpret_cast<float4*>(sH + r * LB + c) =
            kt + r < p.dk ? *reinterpret_cast<const float4*>(hs + (size_t)(kt + r) * p.dv + c0 + c)
                          : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      __syncthreads();
      warp_mma<1, 2, false, false, kSplit>(acc, sQ + kt, LQ, sH, LB, mv, nv, KT);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[0][j][e] *= se[f.row(mv, 0, e)];
    tU.put<LB>(sV);
    __syncthreads();
    warp_mma<1, 2, false, false, kSplit>(acc, sP, LC, sV, LB, mv, nv, C);
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const int m = f.row(mv, 0, e), c = f.col(nv, j, e);
        if (t0 + m < Tn)
          store2(o + ((bT + t0 + m) * p.H + h) * p.dv + c0 + c, acc[0][j][e], acc[0][j][e + 1]);
      }
  }
}

// ---------------------------------------------------------------------------
// 3. per chunk: every gradient
// ---------------------------------------------------------------------------
constexpr int kGradSmemFloats = 2 * C * LC + 4 * C * LB + 2 * KT * LT + 7 * C + 8 * C + 32;

template <typename Tin>
__global__ void __launch_bounds__(NT, 2) bwd_grads_kernel(const BwdParams p) {
  constexpr bool kSplit = sizeof(Tin) == 4;
  extern __shared__ float sm[];
  float* sPE = sm;                  // C x LC  dP e^{G_i - G_j} (lower, with diagonal)
  float* sAE = sPE + C * LC;        // C x LC  dA e^{G_i - G_j} (strictly lower)
  float* s1 = sAE + C * LC;         // C x 32 tiles (stride LT, or LB for the dQ / dK products)
  float* s2 = s1 + C * LB;
  float* s3 = s2 + C * LB;
  float* s4 = s3 + C * LB;
  float* sH = s4 + C * LB;          // KT x LT  h tile      [dk row][dv col]
  float* sD = sH + KT * LT;         // KT x LT  dh_out tile
  float* sG = sD + KT * LT;
  float* se = sG + C; float* sd = se + C; float* sb = sd + C; float* sbe = sb + C;
  float* sdG = sbe + C; float* sdB = sdG + C;
  float* sRg = sdB + C;             // [2][C] row partials of the two column halves
  float* sRb = sRg + 2 * C;         // [2][C]
  float* sRc = sRb + 2 * C;         // [4][C] column partials of the four row blocks
  float* sred = sRc + 4 * C;        // [8]
  const Tin* q = static_cast<const Tin*>(p.q);
  const Tin* k = static_cast<const Tin*>(p.k);
  const Tin* v = static_cast<const Tin*>(p.v);
  const Tin* dO = static_cast<const Tin*>(p.dO);
  const int gc = blockIdx.x, h = blockIdx.y, sq = seq_of_chunk(p, gc);
  if (sq < 0) return;   // past the last chunk (packed sequences)
  const SeqSpan sp = seq_span(p, sq);
  const int n = gc - sp.cfirst, Tn = sp.len;
  const int hq = h * p.Hk / p.H, t0 = n * C, tid = threadIdx.x, w = tid >> 5;
  const size_t bT = sp.tok0;
  const size_t row0 = ((size_t)gc * p.H + h) * C;
  const Frag f;
  const int mq = (w >> 1) * 16, nq = (w & 1) * 32;   // C x C products
  const int mw = (w >> 1) * 16, nw = (w & 1) * 16;   // C x 32 products
  const bool grouped = p.Hk != p.H;
  chunk_gates(p, bT, Tn, h, t0, sG, se, sd, sb, sbe);
  if (tid < C) { sdG[tid] = 0.f; sdB[tid] = 0.f; }

  // A. dO V'^T and dX V'^T over dv tiles; rowsum(dX o V); dV = beta dX
  float aP[1][4][4], aA[1][4][4];
  zero(aP); zero(aA);
  Tin* dv_out = static_cast<Tin*>(p.dv_out);
  // every tile loop below fetches its next tiles before the current products
  TokenTile<VT, Tin> tO, tV;
  BlockTile<VT> tX, tP;
  tO.fetch(dO, bT, t0, Tn, p.H, h, p.dv, 0);
  tX.fetch(p.YX + row0 * p.dv, p.dv, 0);
  tP.fetch(p.UV + row0 * p.dv, p.dv, 0);
  tV.fetch(v, bT, t0, Tn, p.H, h, p.dv, 0);
  for (int c0 = 0; c0 < p.dv; c0 += VT) {
    __syncthreads();
    tO.put<LT>(s1, nullptr);
    tX.put<LT>(s2);
    tP.put<LT>(s3);
    tV.put<LT>(s4, nullptr);
    __syncthreads();
    if (c0 + VT < p.dv) {
      tO.fetch(dO, bT, t0, Tn, p.H, h, p.dv, c0 + VT);
      tX.fetch(p.YX + row0 * p.dv, p.dv, c0 + VT);
      tP.fetch(p.UV + row0 * p.dv, p.dv, c0 + VT);
      tV.fetch(v, bT, t0, Tn, p.H, h, p.dv, c0 + VT);
    }
    warp_mma<1, 4, false, true, kSplit>(aP, s1, LT, s3, LT, mq, nq, VT);
    warp_mma<1, 4, false, true, kSplit>(aA, s2, LT, s3, LT, mq, nq, VT);
    // one warp per row: 32 columns
    for (int q8 = 0; q8 < C * VT / NT; ++q8) {
      const int e = tid + q8 * NT, r = e >> 5, c = e & 31, t = t0 + r;
      const float dx = s2[r * LT + c];
      float part = dx * s4[r * LT + c];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      if (c == 0) sdB[r] += part;
      if (t < Tn) dv_out[((bT + t) * p.H + h) * p.dv + c0 + c] = from_f32<Tin>(sb[r] * dx);
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int m = f.row(mq, 0, e), c = f.col(nq, j, e);
      const float E = c <= m ? gate_exp(sG[m] - sG[c]) : 0.f;
      sPE[m * LC + c] = aP[0][j][e] * E;
      sAE[m * LC + c] = c < m ? -aA[0][j][e] * E : 0.f;
    }

  // B. Q K^T and K K^T; the gate and beta terms through P and A
  float aQK[1][4][4], aKK[1][4][4];
  zero(aQK); zero(aKK);
  TokenTile<KT, Tin> tQ, tK;
  tQ.fetch(q, bT, t0, Tn, p.Hk, hq, p.dk, 0);
  tK.fetch(k, bT, t0, Tn, p.Hk, hq, p.dk, 0);
  for (int c0 = 0; c0 < p.dk; c0 += KT) {
    __syncthreads();
    tQ.put<LT>(s1, nullptr);
    tK.put<LT>(s2, nullptr);
    __syncthreads();
    if (c0 + KT < p.dk) {
      tQ.fetch(q, bT, t0, Tn, p.Hk, hq, p.dk, c0 + KT);
      tK.fetch(k, bT, t0, Tn, p.Hk, hq, p.dk, c0 + KT);
    }
    warp_mma<1, 4, false, true, kSplit>(aQK, s1, LT, s2, LT, mq, nq, KT);
    warp_mma<1, 4, false, true, kSplit>(aKK, s2, LT, s2, LT, mq, nq, KT);
  }
  {
    // rows: quad sums, then the two column halves; columns: sums over the 8
    // quads, then the four row blocks -- each in a fixed order (no atomics)
    float rowg[2] = {0.f, 0.f}, rowb[2] = {0.f, 0.f}, colg[4][2];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      colg[j][0] = 0.f; colg[j][1] = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int m = f.row(mq, 0, e), c = f.col(nq, j, e);
        const float pe = sPE[m * LC + c], ae = sAE[m * LC + c];
        const float x = fmaf(pe, aQK[0][j][e], ae * sb[m] * aKK[0][j][e]);
        rowg[e >> 1] += x;
        colg[j][e & 1] -= x;
        rowb[e >> 1] = fmaf(ae, aKK[0][j][e], rowb[e >> 1]);
      }
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const float rg = quad_sum(rowg[hh]), rb = quad_sum(rowb[hh]);
      if (f.t == 0) {
        sRg[(w & 1) * C + mq + f.g + 8 * hh] = rg;
        sRb[(w & 1) * C + mq + f.g + 8 * hh] = rb;
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int c2 = 0; c2 < 2; ++c2) {
        const float cg = column_sum(colg[j][c2]);
        if (f.g == 0) sRc[(w >> 1) * C + nq + 8 * j + 2 * f.t + c2] = cg;
      }
    __syncthreads();
    if (tid < C) {
      sdG[tid] += (sRg[tid] + sRg[C + tid]) +
                  ((sRc[tid] + sRc[C + tid]) + (sRc[2 * C + tid] + sRc[3 * C + tid]));
      sdB[tid] += sRb[tid] + sRb[C + tid];
    }
  }

  // C. per dk tile: V' dh^T, dO h^T, dX h^T over dv; then dQ, dK and the row terms
  float rG[2] = {0.f, 0.f}, rB[2] = {0.f, 0.f};
  float rGC = 0.f, rHD = 0.f;
  const size_t st0 = ((size_t)gc * p.H + h) * p.dk;
  // h and dh_out tiles (KT rows from kt, VT columns from c0): one 16-byte
  // vector of each per thread
  static_assert(KT * VT == 4 * NT, "one 16-byte vector of h and of dh per thread");
  const int hr = tid >> 3, hc = (tid & 7) * 4;
  float4 hv, dhv;
  auto fetch_state = [&](int kt, int c0) {
    hv = make_float4(0.f, 0.f, 0.f, 0.f);
    dhv = hv;
    if (kt + hr < p.dk) {
      const size_t off = (st0 + kt + hr) * p.dv + c0 + hc;
      hv = *reinterpret_cast<const float4*>(p.hs + off);
      dhv = *reinterpret_cast<const float4*>(p.dhs + off);
    }
  };
  tO.fetch(dO, bT, t0, Tn, p.H, h, p.dv, 0);
  tX.fetch(p.YX + row0 * p.dv, p.dv, 0);
  tP.fetch(p.UV + row0 * p.dv, p.dv, 0);
  fetch_state(0, 0);
  for (int kt = 0; kt < p.dk; kt += KT) {
    float aKd[1][2][4], aQ0[1][2][4], aM[1][2][4];
    zero(aKd); zero(aQ0); zero(aM);
    for (int c0 = 0; c0 < p.dv; c0 += VT) {
      __syncthreads();
      tO.put<LT>(s1, nullptr);
      tX.put<LT>(s2);
      tP.put<LT>(s3);
      *reinterpret_cast<float4*>(sH + hr * LT + hc) = hv;
      *reinterpret_cast<float4*>(sD + hr * LT + hc) = dhv;
      rHD = fmaf(hv.x, dhv.x, fmaf(hv.y, dhv.y, fmaf(hv.z, dhv.z, fmaf(hv.w, dhv.w, rHD))));
      __syncthreads();
      {
        // the next (dk tile, dv tile) pair
        const int nc0 = c0 + VT < p.dv ? c0 + VT : 0, nkt = c0 + VT < p.dv ? kt : kt + KT;
        if (nkt < p.dk) {
          tO.fetch(dO, bT, t0, Tn, p.H, h, p.dv, nc0);
          tX.fetch(p.YX + row0 * p.dv, p.dv, nc0);
          tP.fetch(p.UV + row0 * p.dv, p.dv, nc0);
          fetch_state(nkt, nc0);
        }
      }
      warp_mma<1, 2, false, true, kSplit>(aKd, s3, LT, sD, LT, mw, nw, VT);
      warp_mma<1, 2, false, true, kSplit>(aQ0, s1, LT, sH, LT, mw, nw, VT);
      warp_mma<1, 2, false, true, kSplit>(aM, s2, LT, sH, LT, mw, nw, VT);
    }
    __syncthreads();
    load_tokens<KT, LB>(s1, q, bT, t0, Tn, p.Hk, hq, p.dk, kt, nullptr);
    load_tokens<KT, LB>(s2, k, bT, t0, Tn, p.Hk, hq, p.dk, kt, nullptr);
    load_tokens<KT, LB>(s4, k, bT, t0, Tn, p.Hk, hq, p.dk, kt, sb);
    __syncthreads();
    float aq[1][2][4], ak[1][2][4], ak2[1][2][4];
    zero(aq); zero(ak); zero(ak2);
    warp_mma<1, 2, false, false, kSplit>(aq, sPE, LC, s2, LB, mw, nw, C);
    warp_mma<1, 2, true, false, kSplit>(ak, sPE, LC, s1, LB, mw, nw, C);
    warp_mma<1, 2, true, false, kSplit>(ak, sAE, LC, s4, LB, mw, nw, C);
    warp_mma<1, 2, false, false, kSplit>(ak2, sAE, LC, s2, LB, mw, nw, C);
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const int m = f.row(mw, 0, e), c = f.col(nw, j, e), col = kt + c, t = t0 + m;
        const float em = se[m], dm = sd[m], bm = sb[m], bem = sbe[m];
        float dq[2], dkv[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const float kv = s2[m * LB + c + u], qv = s1[m * LB + c + u];
          const float kd = aKd[0][j][e + u], q0 = aQ0[0][j][e + u], mm = aM[0][j][e + u];
          dq[u] = fmaf(em, q0, aq[0][j][e + u]);
          dkv[u] = dm * kd - bem * mm + ak[0][j][e + u] + bm * ak2[0][j][e + u];
          rG[e >> 1] += -dm * kd * kv + em * q0 * qv - bem * mm * kv;
          rB[e >> 1] -= em * mm * kv;
          rGC = fmaf(dm * kd, kv, rGC);
        }
        if (t < Tn && col < p.dk) {
          if (grouped) {
            const size_t off = ((bT + t) * p.H + h) * p.dk + col;
            store2(p.dqk + off, dq[0], dq[1]);
            store2(p.dqk + (size_t)p.B * p.T * p.H * p.dk + off, dkv[0], dkv[1]);
          } else {
            const size_t off = ((bT + t) * p.Hk + hq) * p.dk + col;
            store2(static_cast<Tin*>(p.dq) + off, dq[0], dq[1]);
            store2(static_cast<Tin*>(p.dk_out) + off, dkv[0], dkv[1]);
          }
        }
      }
  }
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const float rg = quad_sum(rG[hh]), rb = quad_sum(rB[hh]);
    if (f.t == 0) {
      sRg[(w & 1) * C + mw + f.g + 8 * hh] = rg;
      sRb[(w & 1) * C + mw + f.g + 8 * hh] = rb;
    }
  }
  // dG_C = e^gamma <h, dh_out> + sum(d K o V' dh_out^T)
  float x = fmaf(se[C - 1], rHD, rGC);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  if ((tid & 31) == 0) sred[w] = x;
  __syncthreads();
  if (tid < C) {
    sdG[tid] += sRg[tid] + sRg[C + tid];
    sdB[tid] += sRb[tid] + sRb[C + tid];
  }
  __syncthreads();
  if (tid < 32) {
    float y = tid < NT / 32 ? sred[tid] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) y += __shfl_xor_sync(0xffffffffu, y, o);
    // dg = reverse in-chunk cumulative sum of dG, dG_C added at the last
    // position (tokens past T add nothing else), two tokens per lane
    const int l = tid;
    float x0 = sdG[l], x1 = sdG[l + 32] + (l == 31 ? y : 0.f);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y0 = __shfl_down_sync(0xffffffffu, x0, o);
      const float y1 = __shfl_down_sync(0xffffffffu, x1, o);
      if (l + o < 32) { x0 += y0; x1 += y1; }
    }
    x0 += __shfl_sync(0xffffffffu, x1, 0);
    const int ta = t0 + l, tb = t0 + 32 + l;
    if (ta < Tn) {
      p.dg[(bT + ta) * p.H + h] = x0;
      p.dbeta[(bT + ta) * p.H + h] = sdB[l];
    }
    if (tb < Tn) {
      p.dg[(bT + tb) * p.H + h] = x1;
      p.dbeta[(bT + tb) * p.H + h] = sdB[l + 32];
    }
  }
}

// ---------------------------------------------------------------------------
// 4. grouped q/k heads: dq, dk summed over the value heads of each group
// ---------------------------------------------------------------------------
template <typename Tin>
__global__ void bwd_group_kernel(const BwdParams p) {
  const int rep = p.H / p.Hk;
  const size_t total = (size_t)p.B * p.T * p.Hk * p.dk;
  const size_t plane = (size_t)p.B * p.T * p.H * p.dk;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t d = i % p.dk, bt_hk = i / p.dk;
    const size_t hk = bt_hk % p.Hk, bt = bt_hk / p.Hk;
    const size_t src = (bt * p.H + hk * rep) * p.dk + d;
    float sq = 0.f, sk = 0.f;
    for (int r = 0; r < rep; ++r) {
      sq += p.dqk[src + (size_t)r * p.dk];
      sk += p.dqk[plane + src + (size_t)r * p.dk];
    }
    static_cast<Tin*>(p.dq)[i] = from_f32<Tin>(sq);
    static_cast<Tin*>(p.dk_out)[i] = from_f32<Tin>(sk);
  }
}

// Packed sequences: coff[s] = sum over s' < s of the chunks of sequence s'
// (offsets clamped to [0, T] as the forward does), coff[n_seqs] = all chunks.
// Every value is also clamped to NC, the chunks the workspace holds: offsets
// that rise from 0 to T never reach it, and malformed (overlapping) ones then
// lose chunks instead of reaching past the workspace.
// One CTA of 1024 threads, sequences in tiles of 1024.
__global__ void __launch_bounds__(1024) bwd_chunk_offsets_kernel(const int* cu, int n_seqs, int T,
                                                                 int NC, int* coff) {
  __shared__ int warp_incl[32];
  __shared__ int carry;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  if (tid == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < n_seqs; base += 1024) {
    const int s = base + tid;
    int cnt = 0;
    if (s < n_seqs) {
      const int a0 = min(max(cu[s], 0), T);
      const int a1 = min(max(cu[s + 1], a0), T);
      cnt = (a1 - a0 + C - 1) / C;
    }
    int x = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_incl[w] = x;
    __syncthreads();
    if (w == 0) {
      int y = warp_incl[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int z = __shfl_up_sync(0xffffffffu, y, o);
        if (lane >= o) y += z;
      }
      warp_incl[lane] = y;
    }
    __syncthreads();
    const int incl = carry + (w ? warp_incl[w - 1] : 0) + x;
    if (s < n_seqs) coff[s] = min(incl - cnt, NC);
    __syncthreads();
    if (tid == 1023) carry = incl;
    __syncthreads();
  }
  if (tid == 0) coff[n_seqs] = min(carry, NC);
}

// Workspace: offsets in floats, each array on a 256-byte boundary.
struct WsLayout {
  size_t W, Z, UV, YX, hs, dhs, dqk, coff, tiles, total;
  bool has_tiles;
};

int padded_dk(int dk) { return dk <= 32 ? 32 : dk <= 64 ? 64 : dk <= 128 ? 128 : 256; }

// NC chunks per head, tokens in all, n_seqs chunk offsets (0: dense).  The
// layout every path fits (fp32 W, Z, U/V', Y/dX, entering states, leaving
// state gradients).
WsLayout ws_layout(size_t NC, size_t tokens, int H, int dk, int dv, int n_seqs) {
  const size_t ldw = (size_t)padded_dk(dk);
  WsLayout L{};
  size_t o = 0;
  auto take = [&](size_t n) { const size_t r = o; o += (n + 63) & ~size_t(63); return r; };
  L.W = take(NC * H * C * ldw);
  L.Z = take(NC * H * C * ldw);
  L.UV = take(NC * H * C * dv);
  L.YX = take(NC * H * C * dv);
  L.hs = take(NC * H * dk * dv);
  L.dhs = take(NC * H * dk * dv);
  L.dqk = take(2 * tokens * H * dk);
  L.coff = take(n_seqs ? (size_t)n_seqs + 1 : 0);
  // dense dk = dv = 128: the preparation's [Z | PT | T] slots for the scan
  // kernels (32 KB per chunk and head) share W's region, which only the
  // warp-level forward pass reads (the two never run in one call)
  L.has_tiles = !n_seqs && dk == 128 && dv == 128;
  L.tiles = L.W;
  L.total = o;
  return L;
}

// The layout of the tcgen05 path's bf16 hand-off (dense, dk = dv = 128), in
// floats: the preparation's [Z | PT | T] slots (32 KB per chunk and head), V'
// and dX as bf16 rows (UV), the entering states as bf16 tiles (hs, 32 KB
// slots), the leaving gradients as bf16 tiles with the dX.v row partials (dhs,
// 36 KB slots), and per value head dq, dk for grouped heads.  Z and YX are
// not used there; they alias W and UV.
WsLayout ws_layout_handoff(size_t NC, size_t tokens, int H, bool grouped) {
  WsLayout L{};
  size_t o = 0;
  auto take = [&](size_t n) { const size_t r = o; o += (n + 63) & ~size_t(63); return r; };
  L.W = take(NC * H * (kTileBytesBwdSlot / sizeof(float)));
  L.Z = L.W;
  L.UV = take(NC * H * C * 128);
  L.YX = L.UV;
  L.hs = take(NC * H * (kHandoffHSlot / sizeof(float)));
  L.dhs = take(NC * H * (kHandoffDhSlot / sizeof(float)));
  L.dqk = take(grouped ? 2 * tokens * H * 128 : 0);
  L.coff = take(0);
  L.has_tiles = true;
  L.tiles = L.W;
  L.total = o;
  return L;
}

// Chunks (an upper bound for packed sequences: sum of ceil(len / C) <= T / C + n_seqs).
size_t chunk_count(const ChunkBwdArgs& a) {
  return a.cu_seqlens ? (size_t)(a.T / C) + (size_t)a.B
                      : (size_t)a.B * (size_t)((a.T + C - 1) / C);
}

// Whether the call takes the tcgen05 path with the bf16 hand-off: bf16, dense,
// dk = dv = 128, none of the backward's kernel overrides set.
bool bwd_handoff(const ChunkBwdArgs& a) {
  const KernelOverrides& ov = a.ov;
  return a.dtype == kBF16 && !a.cu_seqlens && a.dk == 128 && a.dv == 128 &&
         bwd_prep_tc_supported(a.dtype, a.dk, a.dv) &&
         bwd_grads_tc_supported(a.dtype, a.dk, a.dv) && !ov.bwd_prep_warp &&
         !ov.bwd_fwdpass_warp && !ov.bwd_revpass_warp && !ov.bwd_grads_warp;
}

WsLayout ws_layout(const ChunkBwdArgs& a) {
  const size_t tokens = a.cu_seqlens ? (size_t)a.T : (size_t)a.B * a.T;
  if (bwd_handoff(a)) return ws_layout_handoff(chunk_count(a), tokens, a.H, a.Hk != a.H);
  return ws_layout(chunk_count(a), tokens, a.H, a.dk, a.dv, a.cu_seqlens ? a.B : 0);
}

template <typename Tin, int DKP>
cudaError_t launch_bwd_t(const ChunkBwdArgs& a, cudaStream_t st) {
  const WsLayout L = ws_layout(a);
  const bool packed = a.cu_seqlens != nullptr;
  float* ws = static_cast<float*>(a.workspace);
  int* coff = packed ? reinterpret_cast<int*>(ws + L.coff) : nullptr;
  const BwdParams p{a.q, a.k, a.v, a.dO, a.g, a.beta, a.h0, a.dhT, a.dq, a.dk_out, a.dv_out,
                    a.dg, a.dbeta, a.dh0, ws + L.W, ws + L.Z, ws + L.UV, ws + L.YX,
                    ws + L.hs, ws + L.dhs, ws + L.dqk, a.cu_seqlens, coff, packed ? a.B : 0,
                    packed ? 1 : a.B, a.T, a.H, a.Hk, a.dk, a.dv,
                    packed ? 0 : (a.T + C - 1) / C, DKP};
  const int NC = (int)chunk_count(a);
  static std::atomic<int> set_prep[kMaxDevices] = {}, set_states[kMaxDevices] = {},
                          set_grads[kMaxDevices] = {};
  const int prep_bytes = kPrepSmemFloats * (int)sizeof(float);
  const int states_bytes = states_smem_floats<DKP>() * (int)sizeof(float);
  const int grads_bytes = kGradSmemFloats * (int)sizeof(float);
  cudaError_t e = ensure_smem(bwd_prep_kernel<Tin>, prep_bytes, set_prep);
  if (e == cudaSuccess) e = ensure_smem(bwd_states_kernel<Tin, DKP>, states_bytes, set_states);
  if (e == cudaSuccess) e = ensure_smem(bwd_grads_kernel<Tin>, grads_bytes, set_grads);
  if (e != cudaSuccess) return e;
  if (packed) bwd_chunk_offsets_kernel<<<1, 1024, 0, st>>>(a.cu_seqlens, a.B, a.T, NC, coff);
  const KernelOverrides& ov = a.ov;
  // bf16, dk = dv = 128: the per-chunk preparation on tcgen05; on dense rows
  // the two state passes on the scan kernels, fed by the forward's preparation
  // (its [Z | PT | T] slots), with no fp32 W, U, Z, Y at all
  const bool tc_prep = sizeof(Tin) == 2 && bwd_prep_tc_supported(a.dtype, a.dk, a.dv) &&
                       !ov.bwd_prep_warp;
  const bool tc_fwd = tc_prep && !packed && L.has_tiles && !ov.bwd_fwdpass_warp;
  const bool hand = bwd_handoff(a);   // (the layout above is then the compact one)
  const bool tc_rev = tc_fwd && !ov.bwd_revpass_warp;
  unsigned char* tiles = reinterpret_cast<unsigned char*>(ws + L.tiles);
  ChunkArgs fa{};
  fa.q = a.q; fa.k = a.k; fa.v = a.v; fa.g = a.g; fa.beta = a.beta; fa.h0 = a.h0;
  fa.B = a.B; fa.T = a.T; fa.H = a.H; fa.Hk = a.Hk; fa.dk = a.dk; fa.dv = a.dv;
  fa.chunk = C; fa.dtype = a.dtype; fa.semantics = kExact;
  fa.workspace = tiles;
  fa.ws_bytes = (size_t)NC * a.H * C * DKP * sizeof(float);   // W's region
  if (tc_fwd) {
    e = launch_chunk_prepare_bwd(fa, st);
    if (e != cudaSuccess) return e;
  }
  if (tc_prep && !tc_rev) {
    // the warp-level passes' operands: W, U for the forward direction, Z, Y
    // for the reverse
    e = launch_bwd_prep_tc(a.q, a.k, a.v, a.dO, a.g, a.beta, tc_fwd ? nullptr : p.W, p.Z,
                           tc_fwd ? nullptr : p.UV, p.YX, a.cu_seqlens, coff,
                           packed ? a.B : 0, NC, a.B, a.T, a.H, a.Hk, st);
    if (e != cudaSuccess) return e;
  } else if (!tc_prep) {
    bwd_prep_kernel<Tin><<<dim3(NC, a.H), NT, prep_bytes, st>>>(p);
  }
  // the tcgen05 scans hand h and dh to the tcgen05 gradients as bf16 tiles
  const bool tc_grads = tc_prep && bwd_grads_tc_supported(a.dtype, a.dk, a.dv) &&
                        !ov.bwd_grads_warp;
  const bool tiles_hd = hand;
  // the hand-off's bf16 V' and dX rows share the UV region: V' first, then dX
  void* dx_bf16 = reinterpret_cast<__nv_bfloat16*>(p.UV) + (size_t)NC * a.H * C * a.dv;
  if (tc_fwd) {
    e = launch_chunk_scan_bwd(fa, p.hs, p.UV, tiles_hd, st);
    if (e != cudaSuccess) return e;
    if (tc_rev) {
      e = launch_chunk_scan_rev(fa, a.dO, a.dhT, a.dh0, p.YX, p.dhs,
                                tiles_hd ? dx_bf16 : nullptr, a.dv_out, st);
      if (e != cudaSuccess) return e;
    } else {
      BwdParams pr = p;
      pr.rev_only = 1;
      bwd_states_kernel<Tin, DKP><<<dim3(a.dv / VT, a.B * a.H, 1), NT, states_bytes, st>>>(pr);
    }
  } else {
    bwd_states_kernel<Tin, DKP><<<dim3(a.dv / VT, a.B * a.H, 2), NT, states_bytes, st>>>(p);
  }
  if (tc_grads) {
    BwdGradsArgs ga{a.q, a.k, a.v, a.dO, a.g, a.beta, p.UV, p.YX, p.hs, p.dhs,
                    a.dq, a.dk_out, a.dv_out, a.dg, a.dbeta, a.Hk != a.H ? p.dqk : nullptr,
                    a.cu_seqlens, coff, packed ? a.B : 0, NC, a.B, a.T, a.H, a.Hk};
    if (tiles_hd) {
      ga.hb = reinterpret_cast<const unsigned char*>(p.hs);
      ga.dhb = reinterpret_cast<const unsigned char*>(p.dhs);
      ga.vpb = p.UV;
      ga.dxb = dx_bf16;
    }
    e = launch_bwd_grads_tc(ga, st);
    if (e != cudaSuccess) return e;
  } else {
    bwd_grads_kernel<Tin><<<dim3(NC, a.H), NT, grads_bytes, st>>>(p);
  }
  if (a.Hk != a.H) {
    const size_t total = (size_t)p.B * a.T * a.Hk * a.dk;
    const size_t want = (total + 255) / 256, cap = (size_t)8 * device_sm_count();
    bwd_group_kernel<Tin><<<(int)(want < cap ? want : cap), 256, 0, st>>>(p);
  }
  return cudaGetLastError();
}

template <typename Tin>
cudaError_t launch_bwd_dtype(const ChunkBwdArgs& a, cudaStream_t st) {
  switch (padded_dk(a.dk)) {
    case 32: return launch_bwd_t<Tin, 32>(a, st);
    case 64: return launch_bwd_t<Tin, 64>(a, st);
    case 128: return launch_bwd_t<Tin, 128>(a, st);
    default: return launch_bwd_t<Tin, 256>(a, st);
  }
}

// Workspace of the forward on these kernels: W, U -> V', the entering states
// (and, packed sequences, the chunk offsets).  n_seqs == 0: B dense rows.
struct FwdWs {
  size_t W, UV, hs, coff, total;
};

FwdWs fwd_ws_layout(int B, int T, int H, int dk, int dv, int n_seqs) {
  const size_t NC = n_seqs ? (size_t)(T / C) + (size_t)n_seqs
                           : (size_t)B * (size_t)((T + C - 1) / C);
  FwdWs L{};
  size_t o = 0;
  auto take = [&](size_t n) { const size_t r = o; o += (n + 63) & ~size_t(63); return r; };
  L.W = take(NC * H * C * (size_t)padded_dk(dk));
  L.UV = take(NC * H * C * dv);
  L.hs = take(NC * H * (size_t)dk * dv);
  L.coff = take(n_seqs ? (size_t)n_seqs + 1 : 0);
  L.total = o;
  return L;
}

template <typename Tin, int DKP>
cudaError_t launch_fwd_t(const ChunkArgs& a, cudaStream_t st) {
  const bool packed = a.cu_seqlens != nullptr;   // B = n_seqs sequences in one row of T tokens
  const FwdWs L = fwd_ws_layout(a.B, a.T, a.H, a.dk, a.dv, packed ? a.B : 0);
  float* ws = static_cast<float*>(a.workspace);
  int* coff = packed ? reinterpret_cast<int*>(ws + L.coff) : nullptr;
  BwdParams p{a.q, a.k, a.v, nullptr, a.g, a.beta, a.h0, nullptr, nullptr, nullptr, nullptr,
              nullptr, nullptr, nullptr, ws + L.W, nullptr, ws + L.UV, nullptr, ws + L.hs,
              nullptr, nullptr, a.cu_seqlens, coff, packed ? a.B : 0, packed ? 1 : a.B, a.T,
              a.H, a.Hk, a.dk, a.dv, packed ? 0 : (a.T + C - 1) / C, DKP};
  p.hTout = a.hT;
  p.o = a.o;
  const int NC = packed ? a.T / C + a.B : a.B * ((a.T + C - 1) / C);
  static std::atomic<int> set_prep[kMaxDevices] = {}, set_states[kMaxDevices] = {},
                          set_out[kMaxDevices] = {};
  const int prep_bytes = kPrepSmemFloats * (int)sizeof(float);
  const int states_bytes = states_smem_floats<DKP>() * (int)sizeof(float);
  const int out_bytes = out_smem_floats<DKP>() * (int)sizeof(float);
  cudaError_t e = ensure_smem(bwd_prep_kernel<Tin>, prep_bytes, set_prep);
  if (e == cudaSuccess) e = ensure_smem(bwd_states_kernel<Tin, DKP>, states_bytes, set_states);
  if (e == cudaSuccess) e = ensure_smem(fwd_out_kernel<Tin, DKP>, out_bytes, set_out);
  if (e != cudaSuccess) return e;
  if (packed) bwd_chunk_offsets_kernel<<<1, 1024, 0, st>>>(a.cu_seqlens, a.B, a.T, NC, coff);
  bwd_prep_kernel<Tin><<<dim3(NC, a.H), NT, prep_bytes, st>>>(p);
  bwd_states_kernel<Tin, DKP><<<dim3(a.dv / VT, a.B * a.H, 1), NT, states_bytes, st>>>(p);
  fwd_out_kernel<Tin, DKP><<<dim3(NC, a.H), NT, out_bytes, st>>>(p);
  return cudaGetLastError();
}

template <typename Tin>
cudaError_t launch_fwd_dtype(const ChunkArgs& a, cudaStream_t st) {
  switch (padded_dk(a.dk)) {
    case 32: return launch_fwd_t<Tin, 32>(a, st);
    case 64: return launch_fwd_t<Tin, 64>(a, st);
    case 128: return launch_fwd_t<Tin, 128>(a, st);
    default: return launch_fwd_t<Tin, 256>(a, st);
  }
}

}  // namespace

size_t chunk_bwd_workspace_bytes(int B, int T, int H, int dk, int dv) {
  ChunkBwdArgs a{};   // (fp32: the layout that fits every path)
  a.B = B; a.T = T; a.H = H; a.Hk = H; a.dk = dk; a.dv = dv; a.dtype = kFP32;
  return sizeof(float) * ws_layout(a).total;
}

size_t chunk_bwd_workspace_bytes_for(const ChunkBwdArgs& a) {
  return sizeof(float) * ws_layout(a).total;
}

size_t chunk_bwd_varlen_workspace_bytes(int n_seqs, int T, int H, int dk, int dv) {
  ChunkBwdArgs a{};
  static const int kPacked = 0;   // any non-NULL pointer: the layout of packed sequences
  a.cu_seqlens = &kPacked;
  a.B = n_seqs; a.T = T; a.H = H; a.Hk = H; a.dk = dk; a.dv = dv; a.dtype = kFP32;
  return sizeof(float) * ws_layout(a).total;
}

bool chunk_bwd_supported(const ChunkBwdArgs& a) {
  return a.dk >= 1 && a.dk <= 256 && a.dv >= VT && a.dv % VT == 0 &&
         (long long)a.B * a.H <= 65535;
}

cudaError_t launch_chunk_bwd(const ChunkBwdArgs& a, cudaStream_t st) {
  if (a.B * a.H == 0 || a.T == 0) return cudaSuccess;   // (the caller handles dh0)
  return a.dtype == kBF16 ? launch_bwd_dtype<__nv_bfloat16>(a, st)
                          : launch_bwd_dtype<float>(a, st);
}

bool chunk_fwd_warp_supported(const ChunkArgs& a) {
  return a.semantics == kExact && (a.dtype == kFP32 || a.dtype == kBF16) && a.dk >= 16 &&
         a.dk <= 256 && a.dk % 16 == 0 && a.dv >= VT && a.dv % VT == 0 &&
         (long long)a.B * a.H <= 65535;
}

size_t chunk_fwd_warp_workspace_bytes(int B, int T, int H, int dk, int dv, int n_seqs) {
  return sizeof(float) * fwd_ws_layout(B, T, H, dk, dv, n_seqs).total;
}

cudaError_t launch_chunk_fwd_warp(const ChunkArgs& a, cudaStream_t st) {
  if (a.B * a.H == 0 || a.T == 0) return cudaSuccess;
  return a.dtype == kBF16 ? launch_fwd_dtype<__nv_bfloat16>(a, st)
                          : launch_fwd_dtype<float>(a, st);
}

}  // namespace gdn
