// C ABI of libgdn_b200.so (declared in include/gdn.h): argument checks on the
// host, then dispatch to the kernels.  No allocation, no CPU fallback.
#include <cstdint>
#include <cstdio>
#include <cstdarg>
#include <cstdlib>
#include <cstring>

#include <atomic>

#include "gdn.h"
#include "gdn_internal.h"

namespace gdn {

namespace {

KernelOverrides read_overrides() {
  KernelOverrides k;
  const char* chunk = getenv("GDN_CHUNK_KERNEL");
  k.chunk_simt = chunk && strcmp(chunk, "simt") == 0;
  k.chunk_fused = chunk && strcmp(chunk, "fused") == 0;
  const char* pair = getenv("GDN_CHUNK_TC_PAIR");
  if (pair && pair[0] == '0') k.tc_pair = 0;
  if (pair && pair[0] == '1') k.tc_pair = 1;
  const char* rec = getenv("GDN_RECURRENT_KERNEL");
  k.recurrent_token = rec && strcmp(rec, "token") == 0;
  const char* pdl = getenv("GDN_DECODE_PDL");
  k.decode_pdl = !(pdl && pdl[0] == '0');
  const char* bprep = getenv("GDN_BWD_PREP");
  k.bwd_prep_warp = bprep && strcmp(bprep, "warp") == 0;
  const char* bfwd = getenv("GDN_BWD_FWDPASS");
  k.bwd_fwdpass_warp = bfwd && strcmp(bfwd, "warp") == 0;
  const char* brev = getenv("GDN_BWD_REVPASS");
  k.bwd_revpass_warp = brev && strcmp(brev, "warp") == 0;
  const char* bgr = getenv("GDN_BWD_GRADS");
  k.bwd_grads_warp = bgr && strcmp(bgr, "warp") == 0;
  return k;
}

// The current choices, packed into one word so that a reload is atomic.
int pack(const KernelOverrides& k) {
  return (k.chunk_simt ? 1 : 0) | (k.chunk_fused ? 2 : 0) | ((k.tc_pair + 1) << 2) |
         (k.recurrent_token ? 16 : 0) | (k.decode_pdl ? 32 : 0) | (k.bwd_prep_warp ? 64 : 0) |
         (k.bwd_fwdpass_warp ? 128 : 0) | (k.bwd_revpass_warp ? 256 : 0) |
         (k.bwd_grads_warp ? 512 : 0);
}

std::atomic<int>& override_word() {
  static std::atomic<int> w{pack(read_overrides())};
  return w;
}

}  // namespace

KernelOverrides kernel_overrides() {
  const int w = override_word().load(std::memory_order_relaxed);
  KernelOverrides k;
  k.chunk_simt = (w & 1) != 0;
  k.chunk_fused = (w & 2) != 0;
  k.tc_pair = ((w >> 2) & 3) - 1;
  k.recurrent_token = (w & 16) != 0;
  k.decode_pdl = (w & 32) != 0;
  k.bwd_prep_warp = (w & 64) != 0;
  k.bwd_fwdpass_warp = (w & 128) != 0;
  k.bwd_revpass_warp = (w & 256) != 0;
  k.bwd_grads_warp = (w & 512) != 0;
  return k;
}

}  // namespace gdn

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool dk_supported(int dk) { return dk == 16 || dk == 32 || dk == 64 || dk == 128 || dk == 256; }

int check_common(const void* q, const void* k, const void* v, const float* g, const float* beta,
                 const float* h0, const void* o, const float* hT, int B, int T, int H, int dk,
                 int dv, int dtype) {
  if (B < 0 || T < 0 || H < 0) return fail(GDN_ERR_INVALID, "negative size B=%d T=%d H=%d", B, T, H);
  if (dtype != GDN_DTYPE_FP32 && dtype != GDN_DTYPE_BF16)
    return fail(GDN_ERR_INVALID, "dtype %d is neither GDN_DTYPE_FP32 nor GDN_DTYPE_BF16", dtype);
  if (!dk_supported(dk))
    return fail(GDN_ERR_UNSUPPORTED, "dk=%d not supported (16, 32, 64, 128 or 256)", dk);
  if (dv < 16 || dv > 512 || dv % 16)
    return fail(GDN_ERR_UNSUPPORTED, "dv=%d not supported (multiple of 16 in [16, 512])", dv);
  const long long elems = (long long)B * T * H;
  if (elems * (dk > dv ? dk : dv) > (1LL << 40))
    return fail(GDN_ERR_INVALID, "tensor too large (B*T*H*dim > 2^40)");
  if (elems > 0) {
    if (!q || !k || !v || !g || !beta || !o)
      return fail(GDN_ERR_INVALID, "q, k, v, g, beta and o must be non-NULL");
    const void* ptrs[6] = {q, k, v, g, beta, o};
    const char* names[6] = {"q", "k", "v", "g", "beta", "o"};
    for (int i = 0; i < 6; ++i)
      if (!aligned16(ptrs[i])) return fail(GDN_ERR_INVALID, "%s is not 16-byte aligned", names[i]);
  }
  if (h0 && !aligned16(h0)) return fail(GDN_ERR_INVALID, "h0 is not 16-byte aligned");
  if (hT && !aligned16(hT)) return fail(GDN_ERR_INVALID, "hT is not 16-byte aligned");
  return GDN_OK;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return GDN_OK;
  return fail(GDN_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Grouped heads: q and k carry Hk heads, v / g / beta / state H, with H % Hk == 0.
int check_groups(int H, int Hk) {
  if (Hk < 0) return fail(GDN_ERR_INVALID, "negative Hk=%d", Hk);
  if (H > 0 && (Hk == 0 || H % Hk != 0))
    return fail(GDN_ERR_INVALID, "H=%d value heads is not a multiple of Hk=%d q/k heads", H, Hk);
  return GDN_OK;
}

int recurrent_fwd(const void* q, const void* k, const void* v, const float* g, const float* beta,
                  const float* h0, void* o, float* hT, int B, int T, int H, int Hk, int dk,
                  int dv, int dtype, void* stream) {
  g_err[0] = '\0';
  int rc = check_common(q, k, v, g, beta, h0, o, hT, B, T, H, dk, dv, dtype);
  if (rc) return rc;
  rc = check_groups(H, Hk);
  if (rc) return rc;
  if (T == 0 && (B * H) > 0 && h0 != hT && hT) {
    // Nothing to run but the state must still be carried through.
    cudaError_t e = h0 ? cudaMemcpyAsync(hT, h0, sizeof(float) * (size_t)B * H * dk * dv,
                                         cudaMemcpyDeviceToDevice, (cudaStream_t)stream)
                       : cudaMemsetAsync(hT, 0, sizeof(float) * (size_t)B * H * dk * dv,
                                         (cudaStream_t)stream);
    return cuda_status(e, "gdn_recurrent_fwd (T=0 state copy)");
  }
  // Whole sequences (T >= 64) on the tcgen05 shapes run on the chunked kernel:
  // the same recurrence (exact semantics) computed chunk by chunk on the
  // tensor cores instead of token by token.  Each CTA reads its tile of h0
  // before it writes the same tile of hT, so h0 == hT stays an in-place update.
  // GDN_RECURRENT_KERNEL=token keeps the token loop (kernel cross-checks).
  if (!gdn::kernel_overrides().recurrent_token && T >= 64) {
    gdn::ChunkArgs ca{q, k, v, g, beta, h0, o, hT, B, T, H, dk, dv, 64, dtype,
                      GDN_SEMANTICS_EXACT, nullptr, 0, Hk};
    if (gdn::chunk_tc_supported(ca))
      return cuda_status(gdn::launch_chunk_tc(ca, (cudaStream_t)stream), "gdn_recurrent_fwd");
  }
  gdn::RecurrentArgs a{q, k, v, g, beta, h0, o, hT, B, T, H, dk, dv, dtype, Hk};
  return cuda_status(gdn::launch_recurrent(a, (cudaStream_t)stream), "gdn_recurrent_fwd");
}

int chunk_fwd(const void* q, const void* k, const void* v, const float* g, const float* beta,
              const float* h0, void* o, float* hT, const int* cu_seqlens, int B, int T, int H,
              int Hk, int dk, int dv, int chunk, int dtype, int semantics, void* workspace,
              size_t ws_bytes, void* stream);

int chunk_bwd(const void* q, const void* k, const void* v, const float* g, const float* beta,
              const float* h0, const void* dO, const float* dhT, void* dq, void* dk_out,
              void* dv_out, float* dg, float* dbeta, float* dh0, const int* cu_seqlens, int B,
              int T, int H, int Hk, int dk, int dv, int dtype, void* workspace, size_t ws_bytes,
              void* stream, const char* what);

// Workspace of a chunked forward (n_seqs: packed sequences, B == n_seqs; 0: dense).
size_t chunk_workspace(int B, int T, int H, int dk, int dv, int chunk, int dtype, int semantics,
                       int n_seqs) {
  (void)chunk;   // exact semantics do not depend on the chunk length
  if (B <= 0 || T <= 0 || H <= 0) return 0;
  gdn::ChunkArgs a{};
  a.B = B; a.T = T; a.H = H; a.Hk = H; a.dk = dk; a.dv = dv; a.chunk = 64; a.dtype = dtype;
  a.semantics = semantics;
  const bool tc_shape = dtype == GDN_DTYPE_BF16 && semantics == GDN_SEMANTICS_EXACT &&
                        (dk == 128 || dk == 256) && dv % 64 == 0;
  // dense rows at dk = 128: the two-launch form's per-chunk operands
  if (tc_shape && n_seqs == 0 && gdn::chunk_scan_shape_ok(a))
    return gdn::chunk_scan_workspace_bytes(B, T, H);
  if (tc_shape || !dk_supported(dk) || !gdn::chunk_fwd_warp_supported(a)) return 0;
  return gdn::chunk_fwd_warp_workspace_bytes(B, T, H, dk, dv, n_seqs);
}

// Arguments of the two-phase chunked forward (gdn_chunk_prepare / gdn_chunk_scan):
// bf16, dk = 128, dv a multiple of 64 (v may be NULL for the preparation), dense
// rows, a workspace of gdn_chunk_workspace_bytes(); T > 0 and B * H > 0.
int check_two_phase(const void* q, const void* k, const void* v, const float* g,
                    const float* beta, int B, int T, int H, int Hk, int dk, int dv, int dtype,
                    const void* workspace, size_t ws_bytes) {
  if (B <= 0 || T <= 0 || H <= 0)
    return fail(GDN_ERR_INVALID, "the two-phase form needs B, T, H > 0 (B=%d T=%d H=%d)", B, T, H);
  if (dtype != GDN_DTYPE_BF16 || dk != 128 || dv % 64 || dv <= 0 || dv > 512)
    return fail(GDN_ERR_UNSUPPORTED, "the two-phase form covers bf16 inputs with dk = 128 and "
                "dv a multiple of 64 up to 512 (dtype=%d dk=%d dv=%d)", dtype, dk, dv);
  int rc = check_groups(H, Hk);
  if (rc) return rc;
  if ((long long)B * H > 65535)
    return fail(GDN_ERR_UNSUPPORTED, "B*H=%lld heads exceed 65535", (long long)B * H);
  const void* ptrs[4] = {q, k, g, beta};
  const char* names[4] = {"q", "k", "g", "beta"};
  for (int i = 0; i < 4; ++i) {
    if (!ptrs[i]) return fail(GDN_ERR_INVALID, "%s must be non-NULL", names[i]);
    if (!aligned16(ptrs[i])) return fail(GDN_ERR_INVALID, "%s is not 16-byte aligned", names[i]);
  }
  if (v && !aligned16(v)) return fail(GDN_ERR_INVALID, "v is not 16-byte aligned");
  const size_t need = gdn::chunk_scan_workspace_bytes(B, T, H);
  if (!workspace || ws_bytes < need)
    return fail(GDN_ERR_INVALID, "workspace of %zu bytes needed, %zu given", need, ws_bytes);
  if (!aligned16(workspace)) return fail(GDN_ERR_INVALID, "workspace is not 16-byte aligned");
  return GDN_OK;
}

// The chunked layer form, dense (cu_seqlens NULL: B rows of T tokens) or packed
// (B = n_seqs sequences in one row of T tokens).
int chunk_fwd_layer(const void* q, const void* k, const void* v, const float* a,
                    const float* b, const float* A_log, const float* dt_bias, const float* h0,
                    float* hT, const void* gate, const float* norm_weight, float eps, void* y,
                    const int* cu_seqlens, int B, int T, int H, int Hk, int dk, int dv,
                    int dtype, void* stream) {
  g_err[0] = '\0';
  const int rows = cu_seqlens ? (B > 0 ? 1 : 0) : B;   // rows of the token tensors
  // a, b take the places of g, beta in the common checks (same shapes)
  int rc = check_common(q, k, v, a, b, h0, y, hT, rows, T, H, dk, dv, dtype);
  if (rc) return rc;
  rc = check_groups(H, Hk);
  if (rc) return rc;
  if (T == 0 || (long long)B * H == 0)   // nothing to normalise: carry the state through
    return chunk_fwd(q, k, v, a, b, h0, y, hT, cu_seqlens, B, T, H, Hk, dk, dv, 64, dtype,
                     GDN_SEMANTICS_EXACT, nullptr, 0, stream);
  // dk = dv = 128: one fused launch; the other tensor-core shapes (dk = 256,
  // dv a multiple of 64): the op with the gates formed in its gate warp, then
  // the gated RMSNorm over its output in place.
  const bool fused = dtype == GDN_DTYPE_BF16 && dk == 128 && dv == 128;
  if (dtype != GDN_DTYPE_BF16 || (dk != 128 && dk != 256) || dv % 64)
    return fail(GDN_ERR_UNSUPPORTED, "the chunked layer form covers bf16 inputs with dk = 128 "
                "or 256 and dv a multiple of 64 (dtype=%d dk=%d dv=%d)", dtype, dk, dv);
  if (!A_log || !dt_bias || !norm_weight)
    return fail(GDN_ERR_INVALID, "A_log, dt_bias and norm_weight must be non-NULL");
  if (gate && !aligned16(gate)) return fail(GDN_ERR_INVALID, "gate is not 16-byte aligned");
  if (!(eps >= 0.f) || eps > 1.f) return fail(GDN_ERR_INVALID, "eps=%g outside [0, 1]", (double)eps);
  gdn::ChunkArgs ca{q, k, v, a, b, h0, y, hT, B, T, H, dk, dv, 64, dtype, GDN_SEMANTICS_EXACT,
                    nullptr, 0, Hk, cu_seqlens};
  if (!gdn::chunk_tc_supported(ca))
    return fail(GDN_ERR_UNSUPPORTED, "the tensor-core chunk kernel is unavailable on this device");
  gdn::LayerArgs la;
  la.a = a; la.b = b; la.A_log = A_log; la.dt_bias = dt_bias;
  la.gate = gate; la.weight = norm_weight; la.eps = eps;
  if (fused)
    return cuda_status(gdn::launch_chunk_tc_layer(ca, la, (cudaStream_t)stream),
                       "gdn_chunk_fwd_layer");
  cudaError_t e = gdn::launch_chunk_tc_gates(ca, la, (cudaStream_t)stream);
  if (e == cudaSuccess)
    e = gdn::launch_gated_norm(y, gate, norm_weight, y, (long long)rows * T * H, dv, eps, dtype,
                               (cudaStream_t)stream);
  return cuda_status(e, "gdn_chunk_fwd_layer");
}

}  // namespace

extern "C" {

int gdn_recurrent_fwd(const void* q, const void* k, const void* v, const float* g,
                      const float* beta, const float* h0, void* o, float* hT, int B, int T,
                      int H, int dk, int dv, int dtype, void* stream) {
  return recurrent_fwd(q, k, v, g, beta, h0, o, hT, B, T, H, H, dk, dv, dtype, stream);
}

int gdn_recurrent_fwd_gva(const void* q, const void* k, const void* v, const float* g,
                          const float* beta, const float* h0, void* o, float* hT, int B, int T,
                          int H, int Hk, int dk, int dv, int dtype, void* stream) {
  return recurrent_fwd(q, k, v, g, beta, h0, o, hT, B, T, H, Hk, dk, dv, dtype, stream);
}

int gdn_recurrent_fwd_layer(const void* q, const void* k, const void* v, const float* a,
                            const float* b, const float* A_log, const float* dt_bias,
                            const float* h0, float* hT, const void* gate,
                            const float* norm_weight, float eps, void* y, int B, int T, int H,
                            int Hk, int dk, int dv, int dtype, void* stream) {
  g_err[0] = '\0';
  // a, b take the places of g, beta in the common checks (same shapes)
  int rc = check_common(q, k, v, a, b, h0, y, hT, B, T, H, dk, dv, dtype);
  if (rc) return rc;
  rc = check_groups(H, Hk);
  if (rc) return rc;
  if (T == 0 || (long long)B * H == 0)   // nothing to normalise: carry the state through
    return recurrent_fwd(q, k, v, a, b, h0, y, hT, B, T, H, Hk, dk, dv, dtype, stream);
  if (!A_log || !dt_bias || !norm_weight)
    return fail(GDN_ERR_INVALID, "A_log, dt_bias and norm_weight must be non-NULL");
  if (!aligned16(norm_weight)) return fail(GDN_ERR_INVALID, "norm_weight is not 16-byte aligned");
  if (gate && !aligned16(gate)) return fail(GDN_ERR_INVALID, "gate is not 16-byte aligned");
  if (!(eps >= 0.f) || eps > 1.f) return fail(GDN_ERR_INVALID, "eps=%g outside [0, 1]", (double)eps);
  if (!gdn::gated_norm_supported(dv, dtype))
    return fail(GDN_ERR_UNSUPPORTED, "the layer form's norm takes dv a multiple of 8 (bf16) or "
                "4 (fp32) up to 1024 / 512 (dv=%d)", dv);
  gdn::LayerArgs la;
  la.a = a; la.b = b; la.A_log = A_log; la.dt_bias = dt_bias;
  la.gate = gate; la.weight = norm_weight; la.eps = eps;
  // Single-token decode at dk = dv = 128: one fused launch.
  if (T == 1 && dk == 128 && dv == 128) {
    gdn::RecurrentArgs ra{q, k, v, nullptr, nullptr, h0, y, hT, B, T, H, dk, dv, dtype, Hk};
    return cuda_status(gdn::launch_recurrent_bulk_layer(ra, la, (cudaStream_t)stream),
                       "gdn_recurrent_fwd_layer");
  }
  // Whole sequences on the tensor-core shapes: the chunked layer form (the
  // same recurrence, as gdn_recurrent_fwd does for the op).
  if (T >= 64 && dtype == GDN_DTYPE_BF16 && (dk == 128 || dk == 256) && dv % 64 == 0)
    return chunk_fwd_layer(q, k, v, a, b, A_log, dt_bias, h0, hT, gate, norm_weight, eps, y,
                           nullptr, B, T, H, Hk, dk, dv, dtype, stream);
  // Otherwise the general recurrent kernel with the gates formed per token,
  // then the gated RMSNorm over its output in place.
  gdn::RecurrentArgs ra{q, k, v, a, b, h0, y, hT, B, T, H, dk, dv, dtype, Hk};
  cudaError_t e = gdn::launch_recurrent_gates(ra, la, (cudaStream_t)stream);
  if (e == cudaSuccess)
    e = gdn::launch_gated_norm(y, gate, norm_weight, y, (long long)B * T * H, dv, eps, dtype,
                               (cudaStream_t)stream);
  return cuda_status(e, "gdn_recurrent_fwd_layer");
}

int gdn_chunk_fwd_layer(const void* q, const void* k, const void* v, const float* a,
                        const float* b, const float* A_log, const float* dt_bias,
                        const float* h0, float* hT, const void* gate, const float* norm_weight,
                        float eps, void* y, int B, int T, int H, int Hk, int dk, int dv,
                        int dtype, void* stream) {
  return chunk_fwd_layer(q, k, v, a, b, A_log, dt_bias, h0, hT, gate, norm_weight, eps, y,
                         nullptr, B, T, H, Hk, dk, dv, dtype, stream);
}

int gdn_chunk_fwd_layer_varlen(const void* q, const void* k, const void* v, const float* a,
                               const float* b, const float* A_log, const float* dt_bias,
                               const float* h0, float* hT, const void* gate,
                               const float* norm_weight, float eps, void* y,
                               const int* cu_seqlens, int n_seqs, int T, int H, int Hk, int dk,
                               int dv, int dtype, void* stream) {
  g_err[0] = '\0';
  if (n_seqs < 0) return fail(GDN_ERR_INVALID, "negative n_seqs=%d", n_seqs);
  if (n_seqs > 0 && !cu_seqlens) return fail(GDN_ERR_INVALID, "cu_seqlens must be non-NULL");
  if (cu_seqlens && (reinterpret_cast<uintptr_t>(cu_seqlens) & 3u))
    return fail(GDN_ERR_INVALID, "cu_seqlens is not 4-byte aligned");
  return chunk_fwd_layer(q, k, v, a, b, A_log, dt_bias, h0, hT, gate, norm_weight, eps, y,
                         cu_seqlens, n_seqs, T, H, Hk, dk, dv, dtype, stream);
}

// Non-zero for the calls that run on the warp-level tensor-core kernels (exact
// semantics; fp32 inputs, or bf16 shapes outside the tcgen05 kernel's): their
// per-chunk W, U -> V' and entering states.
size_t gdn_chunk_workspace_bytes(int B, int T, int H, int dk, int dv, int chunk, int dtype,
                                 int semantics) {
  return chunk_workspace(B, T, H, dk, dv, chunk, dtype, semantics, 0);
}

size_t gdn_chunk_varlen_workspace_bytes(int n_seqs, int T, int H, int dk, int dv, int chunk,
                                        int dtype, int semantics) {
  return chunk_workspace(n_seqs, T, H, dk, dv, chunk, dtype, semantics, n_seqs);
}

int gdn_chunk_fwd(const void* q, const void* k, const void* v, const float* g, const float* beta,
                  const float* h0, void* o, float* hT, int B, int T, int H, int dk, int dv,
                  int chunk, int dtype, int semantics, void* workspace, size_t ws_bytes,
                  void* stream) {
  return chunk_fwd(q, k, v, g, beta, h0, o, hT, nullptr, B, T, H, H, dk, dv, chunk, dtype,
                   semantics, workspace, ws_bytes, stream);
}

int gdn_chunk_fwd_gva(const void* q, const void* k, const void* v, const float* g,
                      const float* beta, const float* h0, void* o, float* hT, int B, int T, int H,
                      int Hk, int dk, int dv, int chunk, int dtype, int semantics,
                      void* workspace, size_t ws_bytes, void* stream) {
  return chunk_fwd(q, k, v, g, beta, h0, o, hT, nullptr, B, T, H, Hk, dk, dv, chunk, dtype,
                   semantics, workspace, ws_bytes, stream);
}

int gdn_chunk_fwd_varlen(const void* q, const void* k, const void* v, const float* g,
                         const float* beta, const float* h0, void* o, float* hT,
                         const int* cu_seqlens, int n_seqs, int T, int H, int Hk, int dk, int dv,
                         int chunk, int dtype, int semantics, void* workspace, size_t ws_bytes,
                         void* stream) {
  g_err[0] = '\0';
  if (n_seqs < 0) return fail(GDN_ERR_INVALID, "negative n_seqs=%d", n_seqs);
  if (n_seqs > 0 && !cu_seqlens) return fail(GDN_ERR_INVALID, "cu_seqlens must be non-NULL");
  if (cu_seqlens && (reinterpret_cast<uintptr_t>(cu_seqlens) & 3u))
    return fail(GDN_ERR_INVALID, "cu_seqlens is not 4-byte aligned");
  if (semantics != GDN_SEMANTICS_EXACT)
    return fail(GDN_ERR_UNSUPPORTED, "packed sequences take exact semantics only");
  return chunk_fwd(q, k, v, g, beta, h0, o, hT, cu_seqlens, n_seqs, T, H, Hk, dk, dv, chunk,
                   dtype, semantics, workspace, ws_bytes, stream);
}

}  // extern "C"

namespace {

// The backward, dense (cu_seqlens NULL: B sequences of T tokens) or packed
// (B = n_seqs sequences in one row of T tokens).
int chunk_bwd(const void* q, const void* k, const void* v, const float* g, const float* beta,
              const float* h0, const void* dO, const float* dhT, void* dq, void* dk_out,
              void* dv_out, float* dg, float* dbeta, float* dh0, const int* cu_seqlens, int B,
              int T, int H, int Hk, int dk, int dv, int dtype, void* workspace, size_t ws_bytes,
              void* stream, const char* what) {
  const int rows = cu_seqlens ? (B > 0 ? 1 : 0) : B;   // rows of the token tensors
  int rc = check_common(q, k, v, g, beta, h0, dO, dhT, rows, T, H, dk, dv, dtype);
  if (rc) return rc;
  rc = check_groups(H, Hk);
  if (rc) return rc;
  if ((long long)rows * T * H > 0) {
    const void* outs[5] = {dq, dk_out, dv_out, dg, dbeta};
    const char* names[5] = {"dq", "dk", "dv", "dg", "dbeta"};
    for (int i = 0; i < 5; ++i) {
      if (!outs[i]) return fail(GDN_ERR_INVALID, "%s must be non-NULL", names[i]);
      if (!aligned16(outs[i])) return fail(GDN_ERR_INVALID, "%s is not 16-byte aligned", names[i]);
    }
  }
  if (dh0 && !aligned16(dh0)) return fail(GDN_ERR_INVALID, "dh0 is not 16-byte aligned");
  gdn::ChunkBwdArgs a{q, k, v, g, beta, h0, dO, dhT, dq, dk_out, dv_out, dg, dbeta, dh0,
                      B, T, H, Hk, dk, dv, dtype, workspace, ws_bytes};
  a.cu_seqlens = cu_seqlens;
  if (!gdn::chunk_bwd_supported(a))
    return fail(GDN_ERR_UNSUPPORTED, "backward supports dk <= 256, dv a multiple of 32 and "
                "sequences x heads <= 65535 (dk=%d dv=%d)", dk, dv);
  // this call's layout (the compact one of the bf16 hand-off when it applies);
  // the dtype-blind queries give at least as much
  const size_t need = (long long)rows * T * H > 0 ? gdn::chunk_bwd_workspace_bytes_for(a) : 0;
  if (ws_bytes < need || (need && !workspace))
    return fail(GDN_ERR_INVALID, "workspace of %zu bytes needed, %zu given", need, ws_bytes);
  if (need && !aligned16(workspace)) return fail(GDN_ERR_INVALID, "workspace is not 16-byte aligned");
  if (T == 0 || (long long)B * H == 0) {
    // no tokens: the initial state's gradient is that of the final state
    if (dh0 && (long long)B * H > 0) {
      cudaError_t e = dhT ? cudaMemcpyAsync(dh0, dhT, sizeof(float) * (size_t)B * H * dk * dv,
                                            cudaMemcpyDeviceToDevice, (cudaStream_t)stream)
                          : cudaMemsetAsync(dh0, 0, sizeof(float) * (size_t)B * H * dk * dv,
                                            (cudaStream_t)stream);
      return cuda_status(e, what);
    }
    return GDN_OK;
  }
  return cuda_status(gdn::launch_chunk_bwd(a, (cudaStream_t)stream), what);
}

int chunk_fwd(const void* q, const void* k, const void* v, const float* g, const float* beta,
              const float* h0, void* o, float* hT, const int* cu_seqlens, int B, int T, int H,
              int Hk, int dk, int dv, int chunk, int dtype, int semantics, void* workspace,
              size_t ws_bytes, void* stream) {
  g_err[0] = '\0';
  // packed sequences: the token tensors are one row of T tokens, the states B = n_seqs
  int rc = check_common(q, k, v, g, beta, h0, o, hT, cu_seqlens ? (B > 0 ? 1 : 0) : B, T, H, dk,
                        dv, dtype);
  if (rc) return rc;
  rc = check_groups(H, Hk);
  if (rc) return rc;
  if (chunk != 16 && chunk != 32 && chunk != 64)
    return fail(GDN_ERR_UNSUPPORTED, "chunk=%d not supported (16, 32 or 64)", chunk);
  if (semantics != GDN_SEMANTICS_EXACT && semantics != GDN_SEMANTICS_REFERENCE)
    return fail(GDN_ERR_INVALID, "semantics %d unknown", semantics);
  const size_t need =
      chunk_workspace(B, T, H, dk, dv, chunk, dtype, semantics, cu_seqlens ? B : 0);
  // The two-launch form's workspace is optional: a call without it (or with a
  // shorter one) runs the one-launch tensor-core kernel, which needs none.
  const bool scan_shape = need > 0 && !cu_seqlens && dtype == GDN_DTYPE_BF16 &&
                          semantics == GDN_SEMANTICS_EXACT && dk == 128 && dv % 64 == 0;
  const bool have_ws = workspace && ws_bytes >= need;
  if (need && !have_ws && !scan_shape)
    return fail(GDN_ERR_INVALID, "workspace of %zu bytes needed, %zu given", need, ws_bytes);
  if (need && have_ws && !aligned16(workspace))
    return fail(GDN_ERR_INVALID, "workspace is not 16-byte aligned");
  if (T == 0 && (B * H) > 0 && hT && h0 != hT) {
    cudaError_t e = h0 ? cudaMemcpyAsync(hT, h0, sizeof(float) * (size_t)B * H * dk * dv,
                                         cudaMemcpyDeviceToDevice, (cudaStream_t)stream)
                       : cudaMemsetAsync(hT, 0, sizeof(float) * (size_t)B * H * dk * dv,
                                         (cudaStream_t)stream);
    return cuda_status(e, "gdn_chunk_fwd (T=0 state copy)");
  }
  gdn::ChunkArgs a{q, k, v, g, beta, h0, o, hT, B, T, H, dk, dv, chunk, dtype, semantics,
                   workspace, ws_bytes, Hk, cu_seqlens};
  // GDN_CHUNK_KERNEL=simt forces the CUDA-core kernel, =fused the one-launch
  // tensor-core kernel (kernel cross-checks; read once).
  const gdn::KernelOverrides ov = gdn::kernel_overrides();
  const bool simt_only = ov.chunk_simt;
  if (!simt_only && !ov.chunk_fused && scan_shape && have_ws && gdn::chunk_scan_supported(a))
    return cuda_status(gdn::launch_chunk_scan(a, (cudaStream_t)stream), "gdn_chunk_fwd");
  if (!simt_only && gdn::chunk_tc_supported(a))
    return cuda_status(gdn::launch_chunk_tc(a, (cudaStream_t)stream), "gdn_chunk_fwd");
  if (!simt_only && need > 0 && !scan_shape)
    return cuda_status(gdn::launch_chunk_fwd_warp(a, (cudaStream_t)stream), "gdn_chunk_fwd");
  if (gdn::chunk_simt_smem_bytes(a) == 0)
    return fail(GDN_ERR_UNSUPPORTED, "no chunk kernel fits dk=%d dv=%d chunk=%d", dk, dv, chunk);
  return cuda_status(gdn::launch_chunk_simt(a, (cudaStream_t)stream), "gdn_chunk_fwd");
}

}  // namespace

extern "C" {

size_t gdn_chunk_bwd_workspace_bytes(int B, int T, int H, int dk, int dv) {
  if (B <= 0 || T <= 0 || H <= 0 || dk <= 0 || dv <= 0) return 0;
  return gdn::chunk_bwd_workspace_bytes(B, T, H, dk, dv);
}

int gdn_chunk_bwd(const void* q, const void* k, const void* v, const float* g,
                  const float* beta, const float* h0, const void* dO, const float* dhT,
                  void* dq, void* dk_out, void* dv_out, float* dg, float* dbeta, float* dh0,
                  int B, int T, int H, int Hk, int dk, int dv, int dtype, void* workspace,
                  size_t ws_bytes, void* stream) {
  g_err[0] = '\0';
  return chunk_bwd(q, k, v, g, beta, h0, dO, dhT, dq, dk_out, dv_out, dg, dbeta, dh0, nullptr, B,
                   T, H, Hk, dk, dv, dtype, workspace, ws_bytes, stream, "gdn_chunk_bwd");
}

size_t gdn_chunk_bwd_workspace_bytes_for(int B, int T, int H, int Hk, int dk, int dv,
                                         int dtype) {
  if (B <= 0 || T <= 0 || H <= 0 || Hk <= 0 || dk <= 0 || dv <= 0 ||
      (dtype != GDN_DTYPE_FP32 && dtype != GDN_DTYPE_BF16))
    return 0;
  gdn::ChunkBwdArgs a{};
  a.B = B; a.T = T; a.H = H; a.Hk = Hk; a.dk = dk; a.dv = dv; a.dtype = dtype;
  return gdn::chunk_bwd_workspace_bytes_for(a);
}

size_t gdn_chunk_bwd_varlen_workspace_bytes(int n_seqs, int T, int H, int dk, int dv) {
  if (n_seqs <= 0 || T <= 0 || H <= 0 || dk <= 0 || dv <= 0) return 0;
  return gdn::chunk_bwd_varlen_workspace_bytes(n_seqs, T, H, dk, dv);
}

int gdn_chunk_bwd_varlen(const void* q, const void* k, const void* v, const float* g,
                         const float* beta, const float* h0, const void* dO, const float* dhT,
                         void* dq, void* dk_out, void* dv_out, float* dg, float* dbeta,
                         float* dh0, const int* cu_seqlens, int n_seqs, int T, int H, int Hk,
                         int dk, int dv, int dtype, void* workspace, size_t ws_bytes,
                         void* stream) {
  g_err[0] = '\0';
  if (n_seqs < 0) return fail(GDN_ERR_INVALID, "negative n_seqs=%d", n_seqs);
  if (n_seqs > 0 && !cu_seqlens) return fail(GDN_ERR_INVALID, "cu_seqlens must be non-NULL");
  if (cu_seqlens && (reinterpret_cast<uintptr_t>(cu_seqlens) & 3u))
    return fail(GDN_ERR_INVALID, "cu_seqlens is not 4-byte aligned");
  return chunk_bwd(q, k, v, g, beta, h0, dO, dhT, dq, dk_out, dv_out, dg, dbeta, dh0,
                   n_seqs > 0 ? cu_seqlens : nullptr, n_seqs, T, H, Hk, dk, dv, dtype, workspace,
                   ws_bytes, stream, "gdn_chunk_bwd_varlen");
}

int gdn_chunk_bwd_noalloc(const void* q, const void* k, const void* v, const float* g,
                          const float* beta, const float* h0, const void* dO, const float* dhT,
                          void* dq, void* dk_out, void* dv_out, float* dg, float* dbeta,
                          float* dh0, int B, int T, int H, int Hk, int dk, int dv, int dtype,
                          void* stream) {
  // gdn_chunk_bwd with the library's fixed scratch array as its workspace.
  // The size check comes first and touches no device; gdn_chunk_bwd then
  // checks everything else and zeroes the accumulators it uses.
  g_err[0] = '\0';
  const size_t need = gdn_chunk_bwd_workspace_bytes_for(B, T, H, Hk, dk, dv, dtype);
  if (need > GDN_CHUNK_BWD_NOALLOC_SCRATCH_BYTES)
    return fail(GDN_ERR_UNSUPPORTED,
                "these sizes need %zu bytes of backward scratch; the allocation-free entry "
                "point has a fixed %zu (B*H*T too large: use gdn_chunk_bwd with a workspace)",
                need, (size_t)GDN_CHUNK_BWD_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  if (need) {
    const int rc = cuda_status(gdn::chunk_bwd_static_scratch(&scratch),
                               "gdn_chunk_bwd_noalloc (scratch address)");
    if (rc) return rc;
  }
  return gdn_chunk_bwd(q, k, v, g, beta, h0, dO, dhT, dq, dk_out, dv_out, dg, dbeta, dh0, B, T,
                       H, Hk, dk, dv, dtype, scratch,
                       scratch ? (size_t)GDN_CHUNK_BWD_NOALLOC_SCRATCH_BYTES : 0, stream);
}

int gdn_chunk_prepare(const void* q, const void* k, const float* g, const float* beta, int B,
                      int T, int H, int Hk, int dk, int dtype, void* workspace, size_t ws_bytes,
                      void* stream) {
  g_err[0] = '\0';
  int rc = check_two_phase(q, k, nullptr, g, beta, B, T, H, Hk, dk, 64, dtype, workspace,
                           ws_bytes);
  if (rc) return rc;
  gdn::ChunkArgs a{q, k, nullptr, g, beta, nullptr, nullptr, nullptr, B, T, H, dk, 64, 64,
                   dtype, GDN_SEMANTICS_EXACT, workspace, ws_bytes, Hk};
  return cuda_status(gdn::launch_chunk_prepare(a, (cudaStream_t)stream), "gdn_chunk_prepare");
}

int gdn_chunk_scan(const void* q, const void* k, const void* v, const float* g,
                   const float* beta, const float* h0, void* o, float* hT, int B, int T, int H,
                   int Hk, int dk, int dv, int dtype, int transition, const void* workspace,
                   size_t ws_bytes, void* stream) {
  g_err[0] = '\0';
  int rc = check_two_phase(q, k, v, g, beta, B, T, H, Hk, dk, dv, dtype, workspace, ws_bytes);
  if (rc) return rc;
  if (transition != 0 && transition != 1)
    return fail(GDN_ERR_INVALID, "transition must be 0 or 1 (got %d)", transition);
  if (transition && h0)
    return fail(GDN_ERR_INVALID, "with transition, the state starts from [0 | I]: h0 must be NULL");
  if (transition && !hT)
    return fail(GDN_ERR_INVALID, "with transition, hT ([B,H,dk,dv+dk]) must be non-NULL");
  const void* ptrs[3] = {h0, o, hT};
  const char* names[3] = {"h0", "o", "hT"};
  for (int i = 0; i < 3; ++i)
    if (ptrs[i] && !aligned16(ptrs[i]))
      return fail(GDN_ERR_INVALID, "%s is not 16-byte aligned", names[i]);
  gdn::ChunkArgs a{q, k, v, g, beta, h0, o, hT, B, T, H, dk, dv, 64, dtype, GDN_SEMANTICS_EXACT,
                   const_cast<void*>(workspace), ws_bytes, Hk};
  return cuda_status(gdn::launch_chunk_scan_prepared(a, transition != 0, (cudaStream_t)stream),
                     "gdn_chunk_scan");
}

int gdn_fold_states(const float* S, const float* M, const float* h0, float* out, int P, int BH,
                    int dk, int dv, int ld, void* stream) {
  g_err[0] = '\0';
  if (P < 0 || BH < 0) return fail(GDN_ERR_INVALID, "negative P=%d or BH=%d", P, BH);
  if (!gdn::state_fold_supported(dk, dv))
    return fail(GDN_ERR_UNSUPPORTED, "the fold covers dk = 128 and dv a multiple of 32 "
                "(dk=%d dv=%d)", dk, dv);
  if (ld % 4 || ld < dv || ld < dk)
    return fail(GDN_ERR_INVALID, "row stride ld=%d must be a multiple of 4 and >= dv, dk", ld);
  if ((long long)BH > 65535) return fail(GDN_ERR_UNSUPPORTED, "BH=%d exceeds 65535", BH);
  if (BH == 0) return GDN_OK;
  if (!out || (P > 0 && (!S || !M)))
    return fail(GDN_ERR_INVALID, "out (and S, M when P > 0) must be non-NULL");
  const void* ptrs[4] = {S, M, h0, out};
  const char* names[4] = {"S", "M", "h0", "out"};
  for (int i = 0; i < 4; ++i)
    if (ptrs[i] && !aligned16(ptrs[i]))
      return fail(GDN_ERR_INVALID, "%s is not 16-byte aligned", names[i]);
  return cuda_status(gdn::launch_state_fold(S, M, h0, out, P, BH, dk, dv, ld,
                                            (cudaStream_t)stream),
                     "gdn_fold_states");
}

const char* gdn_last_error(void) { return g_err; }

void gdn_reload_kernel_overrides(void) {
  gdn::override_word().store(gdn::pack(gdn::read_overrides()), std::memory_order_relaxed);
}

int gdn_device_error(int clear) {
  // Synchronous: waits for the current device's outstanding work.
  const int a = gdn::device_error_recurrent_bulk(clear != 0);
  const int b = gdn::device_error_chunk_tc(clear != 0);
  const int c = gdn::device_error_chunk_scan(clear != 0);
  const int d = gdn::device_error_bwd_prep(clear != 0);
  const int e = gdn::device_error_bwd_grads(clear != 0);
  return a ? a : (b ? b : (c ? c : (d ? d : e)));
}

int gdn_abi_version(void) { return (1 << 16) | 10; }

int gdn_binary_version(void) { return gdn::chunk_scan_binary_version(); }

int gdn_short_conv_fwd(const void* x, const float* weight, const void* state_in, void* state_out,
                       void* y, int B, int T, int C, int K, int activation, int dtype,
                       void* stream) {
  g_err[0] = '\0';
  if (B < 0 || T < 0 || C < 0) return fail(GDN_ERR_INVALID, "negative size B=%d T=%d C=%d", B, T, C);
  if (dtype != GDN_DTYPE_FP32 && dtype != GDN_DTYPE_BF16)
    return fail(GDN_ERR_INVALID, "dtype %d is neither GDN_DTYPE_FP32 nor GDN_DTYPE_BF16", dtype);
  if (activation != 0 && activation != 1)
    return fail(GDN_ERR_INVALID, "activation %d is neither 0 (none) nor 1 (silu)", activation);
  if (K < 1 || K > gdn::kShortConvMaxK)
    return fail(GDN_ERR_UNSUPPORTED, "kernel size K=%d not supported (1 .. %d)", K,
                gdn::kShortConvMaxK);
  if (B > 65535) return fail(GDN_ERR_UNSUPPORTED, "B=%d exceeds 65535", B);
  if (B == 0 || C == 0) return GDN_OK;
  if (!gdn::short_conv_supported(C, K, dtype))
    return fail(GDN_ERR_UNSUPPORTED, "C=%d channels must be a multiple of %d for this dtype", C,
                dtype == GDN_DTYPE_BF16 ? 8 : 4);
  if ((long long)B * ((long long)T + K) * C > (1LL << 40))
    return fail(GDN_ERR_INVALID, "tensor too large (B*T*C > 2^40)");
  if (!weight || !aligned16(weight))
    return fail(GDN_ERR_INVALID, "weight must be non-NULL and 16-byte aligned");
  if (T > 0 && (!x || !y || !aligned16(x) || !aligned16(y)))
    return fail(GDN_ERR_INVALID, "x and y must be non-NULL and 16-byte aligned");
  if ((state_in && !aligned16(state_in)) || (state_out && !aligned16(state_out)))
    return fail(GDN_ERR_INVALID, "the conv states must be 16-byte aligned");
  if (T == 0) {
    // nothing to convolve; the state still carries through
    if (!state_out || state_out == state_in || K == 1) return GDN_OK;
    const size_t bytes = (size_t)B * (K - 1) * C * (dtype == GDN_DTYPE_BF16 ? 2 : 4);
    cudaError_t e = state_in ? cudaMemcpyAsync(state_out, state_in, bytes,
                                               cudaMemcpyDeviceToDevice, (cudaStream_t)stream)
                             : cudaMemsetAsync(state_out, 0, bytes, (cudaStream_t)stream);
    return cuda_status(e, "gdn_short_conv_fwd (T=0 state copy)");
  }
  return cuda_status(gdn::launch_short_conv(x, weight, state_in, state_out, y, B, T, C, K,
                                            activation, dtype, (cudaStream_t)stream),
                     "gdn_short_conv_fwd");
}

int gdn_gated_rmsnorm_fwd(const void* o, const void* gate, const float* weight, float eps,
                          void* y, long long rows, int dv, int dtype, void* stream) {
  g_err[0] = '\0';
  if (rows < 0 || dv < 0) return fail(GDN_ERR_INVALID, "negative size rows=%lld dv=%d", rows, dv);
  if (dtype != GDN_DTYPE_FP32 && dtype != GDN_DTYPE_BF16)
    return fail(GDN_ERR_INVALID, "dtype %d is neither GDN_DTYPE_FP32 nor GDN_DTYPE_BF16", dtype);
  if (!gdn::gated_norm_supported(dv, dtype))
    return fail(GDN_ERR_UNSUPPORTED, "dv=%d: a multiple of 8 (bf16) or 4 (fp32) up to 1024 / "
                "512", dv);
  if (!(eps >= 0.f) || eps > 1.f) return fail(GDN_ERR_INVALID, "eps=%g outside [0, 1]", (double)eps);
  if (rows == 0) return GDN_OK;
  if (!o || !y || !weight) return fail(GDN_ERR_INVALID, "o, y and weight must be non-NULL");
  if (!aligned16(o) || !aligned16(y) || (gate && !aligned16(gate)))
    return fail(GDN_ERR_INVALID, "o, y and gate must be 16-byte aligned");
  return cuda_status(gdn::launch_gated_norm(o, gate, weight, y, rows, dv, eps, dtype,
                                            (cudaStream_t)stream),
                     "gdn_gated_rmsnorm_fwd");
}

}  // extern "C"
