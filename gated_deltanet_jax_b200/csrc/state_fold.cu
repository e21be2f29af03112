// The hand-off of the sequence-split forward: the states entering every
// segment from the segments' affine summaries, in one launch.
//
// Segment p maps the state entering it to the state leaving it by
// h -> M_p h + S_p (S_p: its end state from a zero start, M_p: its transition;
// both from gdn_chunk_scan's transition columns).  From h_0 this kernel writes
//   out[0] = h_0,  out[p + 1] = M_p out[p] + S_p     (p = 0 .. P - 1)
// for every head, in fp32.  One CTA owns one head and 32 state columns and
// walks the segments in order; M_p is staged transposed in shared memory (the
// next one is fetched into registers while this one is applied), and each
// thread computes a 4 x 4 block of the 128 x 32 product with float4 reads.
// This replaces ~3 log2(P) small batched GEMMs of a host-side prefix scan.
#include <cuda_runtime.h>

#include <atomic>

#include "gdn_internal.h"

namespace gdn {

namespace {

constexpr int FK = 128;      // state rows (dk)
constexpr int FC = 32;       // state columns per CTA
constexpr int kFoldThreads = 256;
constexpr int kFoldSmem = (FK * FK + FK * FC) * 4;  // M^T and the running state

// S and M: [P][BH][FK] rows of `ld` floats (S_p in columns 0 .. dv - 1 of its
// array, M_p in 0 .. FK - 1 of its; the two may interleave in one array, as
// the gathered [S | M] summaries do); h0 [BH][FK][dv] (NULL: zero);
// out [P + 1][BH][FK][dv].
__global__ void __launch_bounds__(kFoldThreads)
state_fold_kernel(const float* __restrict__ S, const float* __restrict__ M,
                  const float* __restrict__ h0, float* __restrict__ out, int P, int BH, int dv,
                  int ld) {
  extern __shared__ float4 fold_smem4[];
  float* Mt = reinterpret_cast<float*>(fold_smem4);  // [j][i] = M[i][j]
  float* st = Mt + FK * FK;                          // [j][c], the state entering the segment
  const int tid = threadIdx.x;
  const int bh = blockIdx.y, c0 = blockIdx.x * FC;
  const int ty = tid >> 3, tx = tid & 7;  // rows 4 ty .. 4 ty + 3, columns 4 tx .. 4 tx + 3
  const size_t sd = (size_t)FK * dv;      // one head's state
  // the state entering segment 0
  for (int e = tid; e < FK * FC / 4; e += kFoldThreads) {
    const int r = e / (FC / 4), c4 = e % (FC / 4);
    const float* src = h0 ? h0 + bh * sd + (size_t)r * dv + c0 + 4 * c4 : nullptr;
    const float4 x = src ? *reinterpret_cast<const float4*>(src) : make_float4(0.f, 0.f, 0.f, 0.f);
    *reinterpret_cast<float4*>(st + r * FC + 4 * c4) = x;
    *reinterpret_cast<float4*>(out + bh * sd + (size_t)r * dv + c0 + 4 * c4) = x;
  }
  // M_p in registers: thread tid holds row i = tid % 128, columns 8 jj .. 8 jj + 7
  // for jj = tid / 128 + 2 u (u < 8): one 32-byte sector per load, and the
  // transposed stores of a warp fall on 32 consecutive words of Mt.
  float4 mreg[2 * FK / 16];
  auto fetch = [&](int p) {
    const float* row = M + (((size_t)p * BH + bh) * FK + (tid & (FK - 1))) * ld;
#pragma unroll
    for (int u = 0; u < FK / 16; ++u) {
      const int jj = (tid >> 7) + 2 * u;
      mreg[2 * u] = *reinterpret_cast<const float4*>(row + 8 * jj);
      mreg[2 * u + 1] = *reinterpret_cast<const float4*>(row + 8 * jj + 4);
    }
  };
  if (P > 0) fetch(0);
  for (int p = 0; p < P; ++p) {
    __syncthreads();  // the previous product has read Mt (and st is complete)
#pragma unroll
    for (int u = 0; u < FK / 16; ++u) {
      const int i = tid & (FK - 1), j = 8 * ((tid >> 7) + 2 * u);
      const float4 a = mreg[2 * u], b = mreg[2 * u + 1];
      Mt[(j + 0) * FK + i] = a.x;
      Mt[(j + 1) * FK + i] = a.y;
      Mt[(j + 2) * FK + i] = a.z;
      Mt[(j + 3) * FK + i] = a.w;
      Mt[(j + 4) * FK + i] = b.x;
      Mt[(j + 5) * FK + i] = b.y;
      Mt[(j + 6) * FK + i] = b.z;
      Mt[(j + 7) * FK + i] = b.w;
    }
    __syncthreads();
    if (p + 1 < P) fetch(p + 1);
    // acc = M_p st + S_p over this thread's 4 x 4 block
    float acc[4][4];
    const float* Sp = S + ((size_t)p * BH + bh) * FK * ld;
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const float4 x =
          *reinterpret_cast<const float4*>(Sp + (size_t)(4 * ty + a) * ld + c0 + 4 * tx);
      acc[a][0] = x.x; acc[a][1] = x.y; acc[a][2] = x.z; acc[a][3] = x.w;
    }
#pragma unroll 8
    for (int j = 0; j < FK; ++j) {
      const float4 m = *reinterpret_cast<const float4*>(Mt + j * FK + 4 * ty);
      const float4 x = *reinterpret_cast<const float4*>(st + j * FC + 4 * tx);
      const float mv[4] = {m.x, m.y, m.z, m.w}, xv[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[a][c] = fmaf(mv[a], xv[c], acc[a][c]);
    }
    __syncthreads();  // every thread has read st
    float* dst = out + ((size_t)(p + 1) * BH + bh) * sd;
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const float4 x = make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
      *reinterpret_cast<float4*>(st + (4 * ty + a) * FC + 4 * tx) = x;
      *reinterpret_cast<float4*>(dst + (size_t)(4 * ty + a) * dv + c0 + 4 * tx) = x;
    }
  }
}

}  // namespace

bool state_fold_supported(int dk, int dv) { return dk == FK && dv % FC == 0 && dv > 0; }

cudaError_t launch_state_fold(const float* S, const float* M, const float* h0, float* out, int P,
                              int BH, int dk, int dv, int ld, cudaStream_t st) {
  if (BH == 0) return cudaSuccess;
  if (!state_fold_supported(dk, dv) || BH > 65535 || P < 0 || ld % 4 || ld < dv || ld < FK)
    return cudaErrorInvalidValue;
  static std::atomic<int> slot[kMaxDevices] = {};
  cudaError_t e = ensure_smem(state_fold_kernel, kFoldSmem, slot);
  if (e != cudaSuccess) return e;
  state_fold_kernel<<<dim3(dv / FC, BH), kFoldThreads, kFoldSmem, st>>>(S, M, h0, out, P, BH, dv,
                                                                       ld);
  return cudaGetLastError();
}

}  // namespace gdn
