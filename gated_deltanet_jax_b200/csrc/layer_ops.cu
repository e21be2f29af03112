// The layer's elementwise work around the delta-rule op, for the shapes whose
// op kernels do not fuse it (model.py:15-53, 119-153):
//
//   short_conv_kernel   ShortConvolution (model.py:15-40): a causal depthwise
//                       convolution over time, kernel K, no bias, then SiLU,
//                       with an optional state of the K - 1 inputs before the
//                       first token (decode) and the K - 1 last inputs out;
//   gated_norm_kernel   FusedRMSNormGated (model.py:41-53) over the op's output:
//                       y = o rsqrt(mean(o^2) + eps) w silu(gate), in place.
//
// Both are HBM-bound: each element is read once and written once.  A thread
// owns one 16-byte vector of channels (8 bf16 or 4 fp32), so a warp moves 512
// contiguous bytes per access.
#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {

namespace {

template <typename Tin>
struct Vec16;
template <>
struct Vec16<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ static void load(const __nv_bfloat16* p, float (&f)[N]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 x = __bfloat1622float2(h[i]);
      f[2 * i] = x.x;
      f[2 * i + 1] = x.y;
    }
  }
  __device__ static void store(__nv_bfloat16* p, const float (&f)[N]) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
  }
};
template <>
struct Vec16<float> {
  static constexpr int N = 4;
  __device__ static void load(const float* p, float (&f)[N]) {
    const float4 x = *reinterpret_cast<const float4*>(p);
    f[0] = x.x; f[1] = x.y; f[2] = x.z; f[3] = x.w;
  }
  __device__ static void store(float* p, const float (&f)[N]) {
    *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
  }
};

__device__ __forceinline__ float silu_acc(float x) { return x / (1.f + expf(-x)); }

constexpr int kConvThreads = 128;

// x, y [B, T, C]; w [K, C] fp32 (the flax kernel (K, 1, C) as stored);
// state_in / state_out [B, K - 1, C] in x's dtype (NULL: zeros / not wanted).
// Block (channel vectors, b, token tile of TT).  The K - 1 inputs before the
// tile are read as its halo (from the state before token 0); the tile then
// slides a register window.  The last tile writes the final K - 1 inputs.
template <typename Tin, int K>
__global__ void __launch_bounds__(kConvThreads)
short_conv_kernel(const Tin* __restrict__ x, const float* __restrict__ w,
                  const Tin* state_in, Tin* state_out, Tin* __restrict__ y, int T, int C,
                  int TT, int act) {
  using V = Vec16<Tin>;
  constexpr int N = V::N;
  const int c = (blockIdx.x * kConvThreads + threadIdx.x) * N;
  if (c >= C) return;
  const int b = blockIdx.y;
  const int t0 = blockIdx.z * TT;
  const int t1 = min(T, t0 + TT);
  float wk[K][N];
#pragma unroll
  for (int j = 0; j < K; ++j)
#pragma unroll
    for (int e = 0; e < N; e += 4) {
      const float4 q = *reinterpret_cast<const float4*>(w + (size_t)j * C + c + e);
      wk[j][e] = q.x; wk[j][e + 1] = q.y; wk[j][e + 2] = q.z; wk[j][e + 3] = q.w;
    }
  const Tin* xb = x + (size_t)b * T * C + c;
  // win[j] = input at token t - (K - 1) + j for the next output t
  float win[K > 1 ? K - 1 : 1][N];
#pragma unroll
  for (int j = 0; j < K - 1; ++j) {
    const int tt = t0 - (K - 1) + j;
    if (tt >= 0) {
      V::load(xb + (size_t)tt * C, win[j]);
    } else if (state_in) {
      V::load(state_in + ((size_t)b * (K - 1) + (K - 1) + tt) * C + c, win[j]);
    } else {
#pragma unroll
      for (int e = 0; e < N; ++e) win[j][e] = 0.f;
    }
  }
  for (int t = t0; t < t1; ++t) {
    float cur[N], out[N];
    V::load(xb + (size_t)t * C, cur);
#pragma unroll
    for (int e = 0; e < N; ++e) {
      float acc = wk[K - 1][e] * cur[e];
#pragma unroll
      for (int j = 0; j < K - 1; ++j) acc = fmaf(wk[j][e], win[j][e], acc);
      out[e] = act ? silu_acc(acc) : acc;
    }
    V::store(y + ((size_t)b * T + t) * C + c, out);
#pragma unroll
    for (int j = 0; j + 1 < K - 1; ++j)
#pragma unroll
      for (int e = 0; e < N; ++e) win[j][e] = win[j + 1][e];
    if constexpr (K > 1) {
#pragma unroll
      for (int e = 0; e < N; ++e) win[K - 2][e] = cur[e];
    }
  }
  if (state_out && blockIdx.z == gridDim.z - 1) {
#pragma unroll
    for (int j = 0; j < K - 1; ++j) V::store(state_out + ((size_t)b * (K - 1) + j) * C + c, win[j]);
  }
}

// One warp per row of dv elements (rows = tokens x heads): y = o rsqrt(mean(o^2)
// + eps) w (silu(gate) when gate is given).  o and y may be the same array.
constexpr int kNormWarps = 8;
constexpr int kNormMaxVec = 4;  // 16-byte vectors per lane: dv <= 4 * 32 * N

template <typename Tin>
__global__ void __launch_bounds__(kNormWarps * 32)
gated_norm_kernel(const Tin* o, const Tin* __restrict__ gate, const float* __restrict__ wt,
                  Tin* y, long long rows, int dv, float eps) {
  using V = Vec16<Tin>;
  constexpr int N = V::N;
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * kNormWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nvec = dv / N;
  const Tin* orow = o + row * dv;
  float v[kNormMaxVec][N];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kNormMaxVec; ++i) {
    const int cv = lane + 32 * i;
    if (cv < nvec) {
      V::load(orow + cv * N, v[i]);
#pragma unroll
      for (int e = 0; e < N; ++e) ss = fmaf(v[i][e], v[i][e], ss);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float r = rsqrtf(ss / (float)dv + eps);
#pragma unroll
  for (int i = 0; i < kNormMaxVec; ++i) {
    const int cv = lane + 32 * i;
    if (cv < nvec) {
      float gv[N], out[N];
      if (gate) V::load(gate + row * dv + cv * N, gv);
#pragma unroll
      for (int e = 0; e < N; ++e) {
        const float wv = wt[cv * N + e];
        out[e] = v[i][e] * r * wv * (gate ? silu_acc(gv[e]) : 1.f);
      }
      V::store(y + row * dv + cv * N, out);
    }
  }
}

template <typename Tin>
cudaError_t conv_dispatch(const void* x, const float* w, const void* si, void* so, void* y,
                          int B, int T, int C, int K, int TT, int act, cudaStream_t st) {
  constexpr int N = Vec16<Tin>::N;
  const dim3 grid((C / N + kConvThreads - 1) / kConvThreads, B, (T + TT - 1) / TT);
  const Tin* xi = static_cast<const Tin*>(x);
  const Tin* s_in = static_cast<const Tin*>(si);
  Tin* sout = static_cast<Tin*>(so);
  Tin* yo = static_cast<Tin*>(y);
#define GDN_CONV_CASE(KK)                                                                   \
  case KK:                                                                                  \
    short_conv_kernel<Tin, KK><<<grid, kConvThreads, 0, st>>>(xi, w, s_in, sout, yo, T, C, TT, \
                                                              act);                         \
    break;
  switch (K) {
    GDN_CONV_CASE(1)
    GDN_CONV_CASE(2)
    GDN_CONV_CASE(3)
    GDN_CONV_CASE(4)
    GDN_CONV_CASE(5)
    GDN_CONV_CASE(6)
    GDN_CONV_CASE(7)
    GDN_CONV_CASE(8)
    default: return cudaErrorInvalidValue;
  }
#undef GDN_CONV_CASE
  return cudaGetLastError();
}

}  // namespace

bool short_conv_supported(int C, int K, int dtype) {
  const int n = dtype == kBF16 ? 8 : 4;
  return K >= 1 && K <= kShortConvMaxK && C > 0 && C % n == 0;
}

cudaError_t launch_short_conv(const void* x, const float* w, const void* state_in,
                              void* state_out, void* y, int B, int T, int C, int K, int act,
                              int dtype, cudaStream_t st) {
  if (B == 0 || T == 0) return cudaSuccess;
  if (!short_conv_supported(C, K, dtype) || B > 65535) return cudaErrorInvalidValue;
  // Token tiles of 64; a state updated in place is read by the first tile and
  // written by the last, so it takes one tile over all T.
  int TT = 64;
  if (state_in && state_in == state_out) TT = T;
  if ((T + TT - 1) / TT > 65535) TT = (T + 65534) / 65535;
  return dtype == kBF16
             ? conv_dispatch<__nv_bfloat16>(x, w, state_in, state_out, y, B, T, C, K, TT, act, st)
             : conv_dispatch<float>(x, w, state_in, state_out, y, B, T, C, K, TT, act, st);
}

bool gated_norm_supported(int dv, int dtype) {
  const int n = dtype == kBF16 ? 8 : 4;
  return dv > 0 && dv % n == 0 && dv <= kNormMaxVec * 32 * n;
}

cudaError_t launch_gated_norm(const void* o, const void* gate, const float* w, void* y,
                              long long rows, int dv, float eps, int dtype, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  if (!gated_norm_supported(dv, dtype)) return cudaErrorInvalidValue;
  const long long blocks = (rows + kNormWarps - 1) / kNormWarps;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
  if (dtype == kBF16)
    gated_norm_kernel<__nv_bfloat16><<<(unsigned)blocks, kNormWarps * 32, 0, st>>>(
        static_cast<const __nv_bfloat16*>(o), static_cast<const __nv_bfloat16*>(gate), w,
        static_cast<__nv_bfloat16*>(y), rows, dv, eps);
  else
    gated_norm_kernel<float><<<(unsigned)blocks, kNormWarps * 32, 0, st>>>(
        static_cast<const float*>(o), static_cast<const float*>(gate), w,
        static_cast<float*>(y), rows, dv, eps);
  return cudaGetLastError();
}

}  // namespace gdn
