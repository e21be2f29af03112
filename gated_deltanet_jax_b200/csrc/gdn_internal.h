// Internal launch interface shared by the kernels and the C ABI (gdn_capi.cu).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stddef.h>

#include <atomic>

namespace gdn {

// One-time, per-device host set-up of a kernel (shared-memory opt-in, checks
// of its compiled attributes), so that a launch does not repeat it.  The
// set-up is idempotent: two threads racing on a first launch both run it.
constexpr int kMaxDevices = 64;

inline int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) dev = 0;
  return dev;
}

// Shared-memory opt-in of `kernel` to at least `bytes` on the current device.
// `slot` is the caller's per-kernel cache (largest size set so far, per device).
template <typename Kernel>
cudaError_t ensure_smem(Kernel kernel, int bytes, std::atomic<int> (&slot)[kMaxDevices]) {
  const int dev = current_device();
  if (slot[dev].load(std::memory_order_acquire) >= bytes) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) {
    int cur = slot[dev].load(std::memory_order_relaxed);
    while (cur < bytes && !slot[dev].compare_exchange_weak(cur, bytes)) {
    }
  }
  return e;
}

// Number of SMs of the current device (cached per device).
inline int device_sm_count() {
  static std::atomic<int> cache[kMaxDevices] = {};
  const int dev = current_device();
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n <= 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// Kernel choices a test can force for cross-checks, read from the environment
// on the library's first call that consults them and again at each
// gdn_reload_kernel_overrides() (never per call):
//   GDN_CHUNK_KERNEL=simt    the CUDA-core chunk kernel
//   GDN_CHUNK_KERNEL=fused   the one-launch tensor-core chunk kernel (no workspace)
//   GDN_CHUNK_TC_PAIR=0 / 1  its unpaired / paired form
//   GDN_RECURRENT_KERNEL=token  the token loop for whole sequences
//   GDN_DECODE_PDL=0         decode steps without programmatic dependent launch
//   GDN_BWD_PREP=warp        the backward's warp-level per-chunk preparation
//   GDN_BWD_FWDPASS=warp     the backward's forward pass on its warp-level state kernel
//   GDN_BWD_REVPASS=warp     the backward's reverse pass on its warp-level state kernel
//   GDN_BWD_GRADS=warp       the backward's warp-level per-chunk gradients
struct KernelOverrides {
  bool chunk_simt = false;
  bool chunk_fused = false;
  int tc_pair = -1;  // -1: by occupancy
  bool recurrent_token = false;
  bool decode_pdl = true;
  bool bwd_prep_warp = false;
  bool bwd_fwdpass_warp = false;
  bool bwd_revpass_warp = false;
  bool bwd_grads_warp = false;
};
KernelOverrides kernel_overrides();

enum DType : int { kFP32 = 0, kBF16 = 1 };
enum Semantics : int { kExact = 0, kReference = 1 };

struct RecurrentArgs {
  const void* q;
  const void* k;
  const void* v;
  const float* g;
  const float* beta;
  const float* h0;
  void* o;
  float* hT;
  int B, T, H, dk, dv, dtype;
  int Hk;  // heads of q and k (H % Hk == 0); value head h reads q/k head h * Hk / H
};

struct ChunkArgs {
  const void* q;
  const void* k;
  const void* v;
  const float* g;
  const float* beta;
  const float* h0;
  void* o;
  float* hT;
  int B, T, H, dk, dv, chunk, dtype, semantics;
  void* workspace;
  size_t ws_bytes;
  int Hk;  // heads of q and k (H % Hk == 0); value head h reads q/k head h * Hk / H
  // Packed variable-length sequences: B sequences in one row of T tokens, sequence s
  // being tokens [cu_seqlens[s], cu_seqlens[s + 1]) (device array of B + 1); NULL: dense.
  const int* cu_seqlens = nullptr;
};

struct ChunkBwdArgs {
  const void* q;
  const void* k;
  const void* v;
  const float* g;
  const float* beta;
  const float* h0;     // NULL: zero initial state
  const void* dO;      // gradient of o [B,T,H,dv]
  const float* dhT;    // gradient of the final state, NULL: zero
  void* dq;            // [B,T,Hk,dk] input dtype
  void* dk_out;        // [B,T,Hk,dk] input dtype
  void* dv_out;        // [B,T,H,dv] input dtype
  float* dg;           // [B,T,H]
  float* dbeta;        // [B,T,H]
  float* dh0;          // [B,H,dk,dv], NULL: not wanted
  int B, T, H, Hk, dk, dv, dtype;
  void* workspace;
  size_t ws_bytes;
  // Packed sequences: B = n_seqs sequences in one row of T tokens,
  // sequence s = tokens [cu_seqlens[s], cu_seqlens[s + 1]).
  const int* cu_seqlens = nullptr;
  // The kernel overrides this call runs under: one snapshot, taken before its
  // workspace is checked, so that the layout checked is the layout launched.
  KernelOverrides ov = kernel_overrides();
};

size_t chunk_bwd_workspace_bytes(int B, int T, int H, int dk, int dv);   // every path's
size_t chunk_bwd_workspace_bytes_for(const ChunkBwdArgs& a);              // this call's
size_t chunk_bwd_varlen_workspace_bytes(int n_seqs, int T, int H, int dk, int dv);
bool chunk_bwd_supported(const ChunkBwdArgs& a);
cudaError_t launch_chunk_bwd(const ChunkBwdArgs& a, cudaStream_t st);
// Device address of the allocation-free backward's scratch array on the
// current device (looked up on the first call per device, then kept).
cudaError_t chunk_bwd_static_scratch(void** out);

// The layer form of the decode step and of the chunked forward (model.py:136-139
// before the op, :47-53 after it).
struct LayerArgs {
  const float* a = nullptr;         // raw a_proj output [B, T, H]
  const float* b = nullptr;         // raw b_proj output [B, T, H]
  const float* A_log = nullptr;     // [H]
  const float* dt_bias = nullptr;   // [H]
  const void* gate = nullptr;       // [B, T, H, dv] output gate (input dtype), NULL: plain RMSNorm
  const float* weight = nullptr;    // [dv] norm weight
  float eps = 1e-5f;
};

cudaError_t launch_recurrent(const RecurrentArgs& a, cudaStream_t st);
// The general recurrent kernel with the layer's prologue: a.g / a.beta hold the
// raw a_proj / b_proj outputs, la.A_log / la.dt_bias the gate parameters.
cudaError_t launch_recurrent_gates(const RecurrentArgs& a, const LayerArgs& la, cudaStream_t st);

// Decode step (T == 1) with the state streamed by bulk copies (dk = dv = 128).
bool recurrent_bulk_supported(const RecurrentArgs& a);
cudaError_t launch_recurrent_bulk(const RecurrentArgs& a, cudaStream_t st);
cudaError_t launch_recurrent_bulk_layer(const RecurrentArgs& a, const LayerArgs& la,
                                        cudaStream_t st);

// Device error words of the kernel files with bounded waits (0 = none).
int device_error_recurrent_bulk(bool clear);
int device_error_chunk_tc(bool clear);

// The driver's tensor-map encoder (NULL when the driver does not provide it).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn();
// [B, T, H, D] bf16 as a 4-D TMA map (D, H, T, B), boxes of 64 x 1 x 64 x 1
// with 128-byte swizzle; tokens past T read as zero.
bool make_bf16_map_4d(CUtensorMap* m, const void* base, int B, int T, int H, int D);
// [rows, D] fp32 as a 2-D TMA map, boxes of 32 x 32 with 128-byte swizzle (D % 32 == 0).
bool make_f32_map_2d(CUtensorMap* m, const void* base, long long rows, int D);
// [rows, D] bf16 as a 2-D TMA map: boxes of 64 x 64 with 128-byte swizzle
// (swizzled), or 32 x 32 unswizzled (D % 64 == 0).
bool make_bf16_map_2d(CUtensorMap* m, const void* base, long long rows, int D, bool swizzled);

// Tensor-core chunk kernel: bf16, dk = 128 or 256, dv % 64 == 0, chunk = 64, exact.
bool chunk_tc_supported(const ChunkArgs& a);
cudaError_t launch_chunk_tc(const ChunkArgs& a, cudaStream_t st);
// Its layer form (dk = dv = 128, the two column tiles as one cluster of two
// CTAs): the gates
// from the raw projections (a.g / a.beta unused) and the gated RMSNorm of
// every output row, written to a.o.
cudaError_t launch_chunk_tc_layer(const ChunkArgs& a, const LayerArgs& la, cudaStream_t st);
// Its gates-only form (any tcgen05 shape, unpaired): g and beta from the raw
// projections (a.g / a.beta hold them), o as the op writes it.
cudaError_t launch_chunk_tc_gates(const ChunkArgs& a, const LayerArgs& la, cudaStream_t st);

// Two-launch chunked forward (bf16, dk = 128, dv % 64 == 0, exact, dense rows):
// a preparation kernel over every (chunk, head) writes the state-independent
// per-chunk operands into the workspace, then a scan kernel walks the chunks.
bool chunk_scan_shape_ok(const ChunkArgs& a);    // the shapes it takes (no device query)
bool chunk_scan_supported(const ChunkArgs& a);   // ... and the driver can encode TMA maps
size_t chunk_scan_workspace_bytes(int B, int T, int H);
cudaError_t launch_chunk_scan(const ChunkArgs& a, cudaStream_t st);   // both launches
// The two launches on their own: the preparation of (q, k, g, beta) into the
// workspace, and the scan over a prepared workspace (a.o may be NULL; with
// transition, the state -- a.hT, [B,H,dk,dv+dk] -- gains dk columns that start
// from the identity with v = 0, and a.h0 must be NULL).
cudaError_t launch_chunk_prepare(const ChunkArgs& a, cudaStream_t st);
// The same preparation for the backward's scans: 32 KB slots [Z | PT | T] (T = (I + A)^{-1}
// as bf16 rows), a.ws_bytes >= chunk_scan_bwd_tiles_bytes.
cudaError_t launch_chunk_prepare_bwd(const ChunkArgs& a, cudaStream_t st);
size_t chunk_scan_bwd_tiles_bytes(int B, int T, int H);
cudaError_t launch_chunk_scan_prepared(const ChunkArgs& a, bool transition, cudaStream_t st);
// The forward pass of the backward on the scan kernel (bf16, dk = dv = 128, dense rows):
// a.workspace holds the [Z | PT | T] slots of launch_chunk_prepare_bwd; every chunk's
// entering state goes to hs and V' = T X to vp, in the backward's workspace layouts.
// With hs_tiles (the hand-off to the tcgen05 gradients), the entering states go to hs as
// bf16 [dk][64]-column tiles, 128-byte swizzled (kHandoffHSlot per (chunk, head), 16 KB per
// column tile), and V' to vp as bf16 rows [slots C][dv].
cudaError_t launch_chunk_scan_bwd(const ChunkArgs& a, float* hs, float* vp, bool hs_tiles,
                                  cudaStream_t st);
// The backward's reverse pass on the scan kernels (same shapes and slots): dX = PT^T dO + Z dh
// to yx (fp32), every chunk's leaving state gradient to dhs, the initial state's gradient to
// dh0 (NULL: not wanted), from dO and dhT (NULL: zero).  With dxb (the hand-off to the tcgen05
// gradients; dvo and a.v then required): the leaving gradients go to dhs as bf16 tiles
// (kHandoffDhSlot per (chunk, head)), dX to dxb as bf16 rows [slots C][dv], dV = beta dX
// to dvo ([B,T,H,dv] bf16), and each token row's rowsum(dX o v) by 32-column block to the
// dhs slot + 32 KB ([64][4] fp32).
cudaError_t launch_chunk_scan_rev(const ChunkArgs& a, const void* dO, const float* dhT,
                                  float* dh0, float* yx, float* dhs, void* dxb, void* dvo,
                                  cudaStream_t st);
int device_error_chunk_scan(bool clear);
// Compute capability the scan kernel was compiled for (major * 10 + minor), -1 if unknown.
int chunk_scan_binary_version();

// The backward's per-chunk preparation on tcgen05 (chunk_bwd_prep.cu): W, Z, U, Y
// of every (chunk, head) into the backward's fp32 workspace (rows (gc H + h) C of
// global chunk gc, strides dk and dv; W and U skipped when NULL).  bf16, dk = dv =
// 128.  Dense: n_seqs = 0, B rows of T tokens, NC = B ceil(T / 64).  Packed:
// n_seqs sequences in one row of T tokens (cu, n_seqs + 1 device offsets), coff
// their chunk offsets on the device, NC an upper bound of the chunks.
bool bwd_prep_tc_supported(int dtype, int dk, int dv);
cudaError_t launch_bwd_prep_tc(const void* q, const void* k, const void* v, const void* dO,
                               const float* g, const float* beta, float* W, float* Z, float* U,
                               float* Y, const int* cu, const int* coff, int n_seqs, int NC,
                               int B, int T, int H, int Hk, cudaStream_t st);
int device_error_bwd_prep(bool clear);

// The backward's per-chunk gradients on tcgen05 (chunk_bwd_grads.cu): from q, k, v, dO,
// g, beta and the workspace's V' (UV), dX (YX), entering states (hs) and leaving state
// gradients (dhs), the gradients of q, k, v, g, beta (dq, dk straight into the outputs,
// or per value head into dqk [2][rows T][H][dk] fp32 when dqk is not NULL).  bf16,
// dk = dv = 128; dense (n_seqs = 0, B rows) or packed (n_seqs sequences in one row,
// cu / coff on the device); NC the chunks of every row (an upper bound when packed).
// Slots of the backward's bf16 hand-off (bytes per (chunk, head)): the
// preparation's [Z | PT | T]; the entering state h as a bf16 tile [2 column
// tiles][128 key rows][128 B]; the leaving state gradient dh as the same tile,
// then the rows' dX.v partials ([64 tokens][4] fp32) at + 32 KB.
constexpr int kTileBytesBwdSlot = 32768;
constexpr int kHandoffHSlot = 32768;
constexpr int kHandoffDhSlot = 36864;

struct BwdGradsArgs {
  const void* q; const void* k; const void* v; const void* dO;
  const float* g; const float* beta;
  const float* UV; const float* YX; const float* hs; const float* dhs;
  void* dq; void* dk; void* dv; float* dg; float* dbeta; float* dqk;
  const int* cu; const int* coff;
  int n_seqs, NC, B, T, H, Hk;
  // The scans' bf16 hand-off, or NULL (then UV, YX, hs, dhs are read as fp32 and dV is
  // formed here): h and dh tiles (hs / dhs regions, with the rowsum(dX o v) partials at
  // each dhs slot + 32 KB), V' and dX rows; dV was written by the reverse scan.
  const unsigned char* hb = nullptr;
  const unsigned char* dhb = nullptr;
  const void* vpb = nullptr;
  const void* dxb = nullptr;
};
bool bwd_grads_tc_supported(int dtype, int dk, int dv);
cudaError_t launch_bwd_grads_tc(const BwdGradsArgs& a, cudaStream_t st);
int device_error_bwd_grads(bool clear);

// The layer's elementwise work (layer_ops.cu).  Short convolution + SiLU
// (model.py:15-40): x, y [B,T,C], w [K,C] fp32, states [B,K-1,C] in x's dtype;
// C a multiple of 8 (bf16) or 4 (fp32), K <= kShortConvMaxK.
constexpr int kShortConvMaxK = 8;
bool short_conv_supported(int C, int K, int dtype);
cudaError_t launch_short_conv(const void* x, const float* w, const void* state_in,
                              void* state_out, void* y, int B, int T, int C, int K, int act,
                              int dtype, cudaStream_t st);
// Gated RMSNorm (model.py:41-53) over `rows` rows of dv; o and y may alias.
bool gated_norm_supported(int dv, int dtype);
cudaError_t launch_gated_norm(const void* o, const void* gate, const float* w, void* y,
                              long long rows, int dv, float eps, int dtype, cudaStream_t st);

// The sequence split's hand-off: out[0] = h0, out[p + 1] = M_p out[p] + S_p for
// P segments of BH heads (dk = 128, dv % 32 == 0; S, M rows of `ld` floats).
bool state_fold_supported(int dk, int dv);
cudaError_t launch_state_fold(const float* S, const float* M, const float* h0, float* out, int P,
                              int BH, int dk, int dv, int ld, cudaStream_t st);

// The chunked forward on the backward's warp-level tensor-core kernels (exact
// semantics, dk in 16..256, dv % 32 == 0, dense or packed): fp32 inputs, and
// the bf16 shapes the tcgen05 kernel does not take.  Needs a device workspace
// of chunk_fwd_warp_workspace_bytes() (n_seqs: packed sequences, 0: dense).
bool chunk_fwd_warp_supported(const ChunkArgs& a);
size_t chunk_fwd_warp_workspace_bytes(int B, int T, int H, int dk, int dv, int n_seqs);
cudaError_t launch_chunk_fwd_warp(const ChunkArgs& a, cudaStream_t st);

// Portable CUDA-core chunk kernel (any supported shape, fp32 or bf16 inputs).
cudaError_t launch_chunk_simt(const ChunkArgs& a, cudaStream_t st);
// Shared-memory bytes launch_chunk_simt needs for this shape (0 = unsupported).
size_t chunk_simt_smem_bytes(const ChunkArgs& a);

}  // namespace gdn
