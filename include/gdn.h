/*
 * gdn.h -- C ABI of the B200 (sm_100a) gated delta-rule library (libgdn_b200.so).
 *
 * Plain pointers, sizes and an opaque CUDA stream; no framework types.  Every
 * pointer argument is a DEVICE pointer unless stated otherwise.  Tensors are
 * dense row-major in the reference package's layout:
 *
 *   q, k   [B, T, H, dk]     dtype = `dtype` (GDN_DTYPE_BF16 or GDN_DTYPE_FP32)
 *   v, o   [B, T, H, dv]     dtype = `dtype`
 *   g,beta [B, T, H]         float32 (g = log-decay, <= 0 in practice)
 *   h0,hT  [B, H, dk, dv]    float32 (recurrent state; may be NULL; may alias)
 *
 * Supported head dims: dk in {16, 32, 64, 128, 256}; dv a multiple of 16 in
 * [16, 512].  Every pointer must be 16-byte aligned.  Calls are asynchronous
 * on `stream` (a cudaStream_t; NULL = legacy default stream), allocate no
 * memory, and are reentrant: the only global state is a one-time per-device
 * kernel attribute set-up and the thread-local error message.
 *
 * Return value: GDN_OK or one of the GDN_ERR_* codes; gdn_last_error() then
 * returns a message for the calling thread.
 */
#ifndef GDN_B200_H
#define GDN_B200_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GDN_OK 0
#define GDN_ERR_INVALID 1     /* bad shape, pointer, alignment or flag */
#define GDN_ERR_UNSUPPORTED 2 /* valid request outside the built kernels */
#define GDN_ERR_CUDA 3        /* CUDA launch or runtime error */

#define GDN_DTYPE_FP32 0
#define GDN_DTYPE_BF16 1

/* Chunk-path semantics. */
#define GDN_SEMANTICS_EXACT 0     /* the delta-rule recurrence (default) */
#define GDN_SEMANTICS_REFERENCE 1 /* the reference chunk code as written */

/*
 * Fused recurrent gated delta rule over T tokens (T = 1 is one decode step).
 *
 * Replaces the Pallas call of the reference, ops.py:187-219
 * (fused_recurrent_gated_delta_rule_pallas -> fused_recurrent_kernel_simple,
 * ops.py:162-184).  Per (b, h) and token t, with an fp32 state S [dk, dv]:
 *     S <- e^{g_t} S;  u = beta_t (v_t - k_t^T S);  S <- S + k_t u^T;
 *     o_t = S^T q_t
 * h0 == NULL starts from zeros (the reference's only mode, ops.py:168);
 * hT == NULL drops the final state (the reference returns None, ops.py:219).
 * h0 == hT updates the state in place (decode).  Whole sequences (T >= 64)
 * with bf16 inputs, dk = 128 or 256 and dv % 64 == 0 are computed chunk by
 * chunk on the tensor cores: the same recurrence, equal within bf16 rounding.
 */
int gdn_recurrent_fwd(const void* q, const void* k, const void* v,
                      const float* g, const float* beta,
                      const float* h0, void* o, float* hT,
                      int B, int T, int H, int dk, int dv, int dtype,
                      void* stream);

/*
 * Chunked gated delta-rule forward.
 *
 * Replaces chunk_gated_delta_rule_fwd, ops.py:299-346 (with its helpers
 * chunk_local_cumsum :238, chunk_scaled_dot_kkt :249, solve_inv_I_minus_A
 * :271, recompute_w_u :276 and the lax.scan body :322-340).  With
 * GDN_SEMANTICS_EXACT the result equals gdn_recurrent_fwd on the same inputs
 * (to rounding).  `chunk` is the chunk length C (16, 32 or 64).  h0 == NULL
 * starts from zeros (ops.py:318-319); hT == NULL skips the final state
 * (output_final_state=False, ops.py:344-346).  `workspace` / `ws_bytes` may be
 * NULL / 0 when gdn_chunk_workspace_bytes() returns 0.  It is required where
 * the call runs on the warp-level tensor-core kernels (exact semantics with
 * fp32 inputs, or bf16 shapes other than dk = 128 / 256 with dv % 64 == 0).
 * For bf16 with dk = 128 and dv % 64 == 0 (exact semantics) it is optional:
 * with it the call runs in two launches (gdn_chunk_prepare, gdn_chunk_scan),
 * without it (or with a shorter one) in one.
 */
int gdn_chunk_fwd(const void* q, const void* k, const void* v,
                  const float* g, const float* beta,
                  const float* h0, void* o, float* hT,
                  int B, int T, int H, int dk, int dv, int chunk,
                  int dtype, int semantics,
                  void* workspace, size_t ws_bytes, void* stream);

/*
 * Grouped value heads ("GVA"): q and k carry Hk heads, v, g, beta, o and the
 * states carry H heads, H a multiple of Hk; value head h reads q/k head
 * h * Hk / H.  The result equals gdn_recurrent_fwd / gdn_chunk_fwd called on
 * q and k with each head repeated H / Hk times in place -- what the reference
 * layer does with jnp.repeat before calling its ops (model.py:132-135) --
 * without materialising the repeats.  Hk == H is the plain call.
 */
int gdn_recurrent_fwd_gva(const void* q, const void* k, const void* v,
                          const float* g, const float* beta,
                          const float* h0, void* o, float* hT,
                          int B, int T, int H, int Hk, int dk, int dv, int dtype,
                          void* stream);

int gdn_chunk_fwd_gva(const void* q, const void* k, const void* v,
                      const float* g, const float* beta,
                      const float* h0, void* o, float* hT,
                      int B, int T, int H, int Hk, int dk, int dv, int chunk,
                      int dtype, int semantics,
                      void* workspace, size_t ws_bytes, void* stream);

/*
 * The recurrent op with the GatedDeltaNet layer's work on either side of it:
 *   before  beta = sigmoid(b), g = -exp(A_log[h]) * softplus(a + dt_bias[h])
 *           from the raw a_proj / b_proj outputs a, b [B, 1, H] (model.py:136-139);
 *   after   y = o * rsqrt(mean(o^2) + eps) * norm_weight, times silu(gate) when
 *           gate [B, 1, H, dv] (input dtype) is given, over each head's dv
 *           outputs (FusedRMSNormGated, model.py:41-53; gate NULL: the
 *           ungated RMSNorm of model.py:150-151).
 * The recurrent step itself is gdn_recurrent_fwd_gva's (state in / out,
 * h0 == hT in place).  y [B, T, H, dv] in the input dtype; A_log, dt_bias [H]
 * and norm_weight [dv] fp32 (16-byte aligned).  Single-token decode at
 * dk = dv = 128 runs all of it in one kernel.  Other shapes: whole sequences
 * (T >= 64) on the tensor-core shapes take gdn_chunk_fwd_layer; the rest run
 * the general recurrent kernel with the gates formed per token, then the gated
 * RMSNorm (gdn_gated_rmsnorm_fwd) over its output in place (dv a multiple of 8
 * (bf16) or 4 (fp32), up to 512).  No counterpart in the reference, where these
 * are separate jax.numpy operations around the op.
 */
int gdn_recurrent_fwd_layer(const void* q, const void* k, const void* v,
                            const float* a, const float* b,
                            const float* A_log, const float* dt_bias,
                            const float* h0, float* hT,
                            const void* gate, const float* norm_weight, float eps,
                            void* y, int B, int T, int H, int Hk, int dk, int dv,
                            int dtype, void* stream);

/*
 * The chunked forward with the same layer work on either side of it
 * (prefill): gdn_recurrent_fwd_layer's prologue and epilogue around
 * gdn_chunk_fwd_gva (exact semantics), for any T >= 0.  a, b [B, T, H] fp32
 * (raw a_proj / b_proj outputs); gate [B, T, H, dv] (input dtype) or NULL;
 * y [B, T, H, dv] in the input dtype.  Supported: bf16 inputs with dk = 128
 * or 256 and dv a multiple of 64 (GDN_ERR_UNSUPPORTED otherwise; dk = 256,
 * dv = 512 are the reference's default head dims).  At dk = dv = 128 it is one
 * launch, and the RMS statistic is taken over the fp32 outputs before any
 * rounding; at the other shapes the chunk kernel forms the gates itself and
 * writes o into y, and a second launch normalises y in place (the statistic
 * over the bf16 o).  Replaces the separate operations of
 * model.py:136-139 and :147-153 around chunk_gated_delta_rule_fwd
 * (ops.py:299); no single counterpart in the reference.
 */
int gdn_chunk_fwd_layer(const void* q, const void* k, const void* v,
                        const float* a, const float* b,
                        const float* A_log, const float* dt_bias,
                        const float* h0, float* hT,
                        const void* gate, const float* norm_weight, float eps,
                        void* y, int B, int T, int H, int Hk, int dk, int dv,
                        int dtype, void* stream);

/*
 * gdn_chunk_fwd_layer on packed variable-length sequences, laid out as for
 * gdn_chunk_fwd_varlen: n_seqs sequences back to back in one row of T tokens
 * (q, k [1, T, Hk, dk]; v, gate, y [1, T, H, dv]; a, b [1, T, H]), sequence s
 * the tokens [cu_seqlens[s], cu_seqlens[s + 1]); h0 / hT [n_seqs, H, dk, dv].
 * Each sequence gets what gdn_chunk_fwd_layer gives it on its own.  No
 * counterpart in the reference, whose layer takes one dense [B, T] batch.
 */
int gdn_chunk_fwd_layer_varlen(const void* q, const void* k, const void* v,
                               const float* a, const float* b,
                               const float* A_log, const float* dt_bias,
                               const float* h0, float* hT,
                               const void* gate, const float* norm_weight, float eps,
                               void* y, const int* cu_seqlens, int n_seqs,
                               int T, int H, int Hk, int dk, int dv,
                               int dtype, void* stream);

/*
 * Packed variable-length sequences for the chunked forward: n_seqs sequences
 * stored back to back in one row of T tokens -- q, k [1, T, Hk, dk], v, o
 * [1, T, H, dv], g, beta [1, T, H] -- with sequence s the tokens
 * [cu_seqlens[s], cu_seqlens[s + 1]) (cu_seqlens: device int32[n_seqs + 1],
 * non-decreasing from 0 to T; offsets are clamped to [0, T]).  h0 / hT are
 * [n_seqs, H, dk, dv].  Each sequence gets exactly what gdn_chunk_fwd_gva
 * gives it on its own.  The workspace is gdn_chunk_varlen_workspace_bytes().
 * No counterpart in the reference, whose ops take one dense [B, T] batch;
 * exact semantics only.
 */
int gdn_chunk_fwd_varlen(const void* q, const void* k, const void* v,
                         const float* g, const float* beta,
                         const float* h0, void* o, float* hT,
                         const int* cu_seqlens, int n_seqs, int T, int H, int Hk,
                         int dk, int dv, int chunk, int dtype, int semantics,
                         void* workspace, size_t ws_bytes, void* stream);

/*
 * Gradients of the delta-rule forward (the recurrence, i.e. exact semantics)
 * with respect to q, k, v, g, beta and the initial state, given the gradient
 * dO of o and dhT of the final state (NULL = 0).  No counterpart in the
 * reference, which differentiates its chunk path (ops.py:238-346) with JAX
 * autodiff; this is the backward of gdn_chunk_fwd_gva / gdn_recurrent_fwd_gva
 * (ops.py:170-184 with a state carry).  Layouts as the forward's: dq, dk
 * [B,T,Hk,dk] and dv [B,T,H,dv] in the input dtype, dg, dbeta [B,T,H] and dh0
 * [B,H,dk,dv] fp32 (dh0 NULL: not wanted).  Needs dk <= 256 and dv a multiple
 * of 32, and a device workspace of gdn_chunk_bwd_workspace_bytes_for() or
 * gdn_chunk_bwd_workspace_bytes() (per-chunk intermediates: the state entering
 * and the state gradient leaving every chunk, and [T, dk | dv] products per
 * head).  Deterministic: the
 * same inputs give the same bits on every run.
 */
int gdn_chunk_bwd(const void* q, const void* k, const void* v,
                  const float* g, const float* beta, const float* h0,
                  const void* dO, const float* dhT,
                  void* dq, void* dk, void* dv, float* dg, float* dbeta, float* dh0,
                  int B, int T, int H, int Hk, int dk_dim, int dv_dim, int dtype,
                  void* workspace, size_t ws_bytes, void* stream);

/* Device workspace bytes gdn_chunk_bwd needs for these sizes, whatever the
 * dtype and kernels (enough for every path). */
size_t gdn_chunk_bwd_workspace_bytes(int B, int T, int H, int dk, int dv);

/*
 * Device workspace bytes gdn_chunk_bwd needs for exactly this call's sizes,
 * grouped heads and dtype (0 for invalid arguments): at bf16, dk = dv = 128 the
 * tensor-core path hands bf16 tiles between its launches and needs about 40 %
 * of gdn_chunk_bwd_workspace_bytes() (0.55 against 1.34 GB at B=4 T=4096
 * H=16).  Either size is accepted.
 */
size_t gdn_chunk_bwd_workspace_bytes_for(int B, int T, int H, int Hk, int dk, int dv,
                                         int dtype);

/*
 * The backward of gdn_chunk_fwd_varlen: n_seqs sequences packed back to back
 * in one row of T tokens (q, k, dq, dk [1, T, Hk, dk]; v, dO, dv [1, T, H, dv];
 * g, beta, dg, dbeta [1, T, H]; sequence s the tokens [cu_seqlens[s],
 * cu_seqlens[s + 1]), device int32, offsets clamped to [0, T]); h0, dhT, dh0
 * [n_seqs, H, dk, dv].  Every sequence gets what gdn_chunk_bwd gives it on its
 * own.  No counterpart in the reference, whose ops take one dense [B, T]
 * batch; limits as gdn_chunk_bwd's, and the workspace of
 * gdn_chunk_bwd_varlen_workspace_bytes().
 */
int gdn_chunk_bwd_varlen(const void* q, const void* k, const void* v,
                         const float* g, const float* beta, const float* h0,
                         const void* dO, const float* dhT,
                         void* dq, void* dk, void* dv, float* dg, float* dbeta, float* dh0,
                         const int* cu_seqlens, int n_seqs, int T, int H, int Hk,
                         int dk_dim, int dv_dim, int dtype,
                         void* workspace, size_t ws_bytes, void* stream);

/* Device workspace bytes gdn_chunk_bwd_varlen needs for these sizes. */
size_t gdn_chunk_bwd_varlen_workspace_bytes(int n_seqs, int T, int H, int dk, int dv);

/*
 * The backward with no device allocation anywhere: no counterpart in the
 * reference (which has no backward of its own), an addition for callers that
 * cannot allocate device memory and cannot pass gdn_chunk_bwd its workspace --
 * e.g. a custom-call handler inside XLA without access to its scratch allocator
 * (XLA keeps most of HBM in its own pool, so a cudaMalloc there can fail or
 * fragment memory), or a loop that must not stop for cudaMalloc, which can
 * synchronise the whole device.
 *
 * Arguments and results are gdn_chunk_bwd's, without the workspace: the
 * caller still passes every input and output.  The scratch is instead a
 * fixed array of GDN_CHUNK_BWD_NOALLOC_SCRATCH_BYTES (64 MiB) in this
 * library's own device memory; sizes whose gdn_chunk_bwd_workspace_bytes_for()
 * is larger are rejected with GDN_ERR_UNSUPPORTED (e.g. B*H = 16 heads at
 * dk = dv = 128 fit up to T = 1984 tokens in bf16, T = 768 in fp32).  The call itself allocates
 * nothing: no cudaMalloc, cudaFree or allocating library routine.
 *
 * - The array is reserved on a GPU when the driver loads the module that
 *   holds it there, and held until the process exits.  The library keeps that
 *   array in a module of its own (its files are compiled separately, without
 *   relocatable device code), so under CUDA's default lazy loading the 64 MiB
 *   are reserved at the first call of this entry point on a GPU.  With eager
 *   loading (CUDA_MODULE_LOADING=EAGER) every process that loads the library
 *   reserves them on every GPU it initialises, whether or not it calls this.
 * - The first call on each device also finds the array's address and sets up
 *   the kernels; make it before any stream capture.
 * - Every call on a device uses the same array, which keeps the previous
 *   call's contents (the call zeroes what must start at zero).  Calls that
 *   overlap on the GPU -- on different streams, or from different threads --
 *   race on it and give wrong gradients: order them on one stream.
 */
#define GDN_CHUNK_BWD_NOALLOC_SCRATCH_BYTES ((size_t)64 << 20)
int gdn_chunk_bwd_noalloc(const void* q, const void* k, const void* v,
                          const float* g, const float* beta, const float* h0,
                          const void* dO, const float* dhT,
                          void* dq, void* dk, void* dv, float* dg, float* dbeta, float* dh0,
                          int B, int T, int H, int Hk, int dk_dim, int dv_dim, int dtype,
                          void* stream);

/* Device scratch bytes gdn_chunk_fwd takes for these sizes (0 = none; for bf16
 * with dk = 128 and dv % 64 == 0, the two-launch form's, which the call may go
 * without). */
size_t gdn_chunk_workspace_bytes(int B, int T, int H, int dk, int dv, int chunk,
                                 int dtype, int semantics);

/* Device scratch bytes gdn_chunk_fwd_varlen needs for n_seqs packed sequences
 * in one row of T tokens (0 = none).  No counterpart in the reference. */
size_t gdn_chunk_varlen_workspace_bytes(int n_seqs, int T, int H, int dk, int dv, int chunk,
                                        int dtype, int semantics);

/*
 * Device-side error word of the current device (0 = none; 1 = a bounded wait
 * inside a kernel gave up, so that launch's results are invalid).  Kernels
 * with pipelined copies never spin without limit: a wait that runs out
 * records the error and the kernel returns.  Synchronous (it waits for the
 * device's outstanding work); clear != 0 resets the word.  Diagnostics only;
 * no counterpart in the reference, which has no device-side waits.
 */
int gdn_device_error(int clear);

/*
 * The chunked forward's two launches on their own (bf16 inputs, dk = 128, dv a
 * multiple of 64, exact semantics, dense rows): gdn_chunk_prepare computes the
 * per-chunk operands that depend on q, k, g and beta only (the triangular
 * solve of each chunk, ops.py:249-297) into `workspace`
 * (gdn_chunk_workspace_bytes() for this shape); gdn_chunk_scan then runs the
 * sequential scan over chunks (the lax.scan of ops.py:322-341) for any v and
 * initial state, reading that workspace.  gdn_chunk_fwd is the two in a row.
 * A caller that scans the same q, k, g, beta more than once -- the two passes
 * of a sequence split -- prepares once.
 *
 * gdn_chunk_scan: o may be NULL (no output stored).  transition = 1 adds dk
 * state columns that run the same recurrence from the identity with v = 0, so
 * hT ([B,H,dk,dv+dk], required) holds the segment's end state from h0 = 0 and
 * its transition matrix side by side (h0 must then be NULL).  No counterpart
 * in the reference, whose chunk path is one jitted function.
 */
int gdn_chunk_prepare(const void* q, const void* k, const float* g, const float* beta, int B,
                      int T, int H, int Hk, int dk, int dtype, void* workspace, size_t ws_bytes,
                      void* stream);
int gdn_chunk_scan(const void* q, const void* k, const void* v, const float* g,
                   const float* beta, const float* h0, void* o, float* hT, int B, int T, int H,
                   int Hk, int dk, int dv, int dtype, int transition, const void* workspace,
                   size_t ws_bytes, void* stream);

/*
 * The hand-off of a sequence split over P segments: segment p maps the state
 * entering it to S_p + M_p h (its end state from zero and its transition, as
 * gdn_chunk_scan's transition columns give them).  Writes out[0] = h0 (zero if
 * NULL) and out[p + 1] = M_p out[p] + S_p, fp32, for BH heads; dk = 128, dv a
 * multiple of 32.  S and M are [P][BH][dk] rows of `ld` floats (they may
 * interleave in one array: S = base, M = base + dv, ld = dv + dk); h0 is
 * [BH][dk][dv] and out [P + 1][BH][dk][dv].  No counterpart in the reference,
 * which has no sequence split.
 */
int gdn_fold_states(const float* S, const float* M, const float* h0, float* out, int P, int BH,
                    int dk, int dv, int ld, void* stream);

/* Message for the last non-OK return on the calling thread ("" if none). */
const char* gdn_last_error(void);

/*
 * Re-read the kernel-choice variables of the environment (GDN_CHUNK_KERNEL =
 * simt | fused, GDN_CHUNK_TC_PAIR = 0 | 1, GDN_RECURRENT_KERNEL = token,
 * GDN_DECODE_PDL = 0), which the library otherwise reads once, on its first
 * call that consults them.  For cross-checks of one kernel against another in
 * one process; the default choices need none of them.  No counterpart in the
 * reference, which has one kernel per op.
 */
void gdn_reload_kernel_overrides(void);

/*
 * The layer's short convolution (ShortConvolution, model.py:15-40, applied to
 * q, k and v at :119-122): a causal depthwise convolution over time with
 * kernel K (no bias), then SiLU when activation = 1 (0: none):
 *   y[b, t, c] = act(sum_j weight[j, c] * x[b, t - (K - 1) + j, c]),
 * with the inputs before token 0 taken from state_in [B, K - 1, C] (x's
 * dtype; NULL: zeros, the reference's left padding).  state_out [B, K - 1, C]
 * (NULL: not wanted) receives the last K - 1 inputs, for the next decode
 * step; it may be state_in (in place).  x, y [B, T, C] bf16 or fp32; weight
 * [K, C] fp32 (the flax kernel (K, 1, C) as stored).  C a multiple of 8
 * (bf16) or 4 (fp32), K <= 8, 16-byte aligned pointers.  The reference's
 * layer has no conv state (it reruns whole sequences); with state_in = NULL
 * and state_out = NULL this is its call.
 */
int gdn_short_conv_fwd(const void* x, const float* weight, const void* state_in,
                       void* state_out, void* y, int B, int T, int C, int K,
                       int activation, int dtype, void* stream);

/*
 * FusedRMSNormGated (model.py:41-53) over `rows` rows of dv elements:
 * y = o * rsqrt(mean(o^2) + eps) * weight, times silu(gate) when gate (same
 * shape as o) is given.  o, gate, y bf16 or fp32 (dtype); weight [dv] fp32;
 * y may be o (in place).  dv a multiple of 8 (bf16) or 4 (fp32), up to 1024 /
 * 512.
 */
int gdn_gated_rmsnorm_fwd(const void* o, const void* gate, const float* weight, float eps,
                          void* y, long long rows, int dv, int dtype, void* stream);

/* ABI version of this header: (major << 16) | minor (1.3: _gva, _varlen, backward;
 * 1.4: backward of packed sequences, the allocation-free backward;
 * 1.5: the layer form of the decode step; 1.6: the layer form of the chunked
 * forward; 1.7: dk = 256 on the tensor cores, the chunked forward's workspace
 * for fp32 inputs, gdn_chunk_varlen_workspace_bytes; 1.8: the two-launch chunked
 * forward and its workspace (bf16, dk = 128), gdn_chunk_prepare / gdn_chunk_scan,
 * gdn_fold_states,
 * gdn_reload_kernel_overrides, gdn_binary_version; 1.9: the layer forms at
 * the other tensor-core shapes and the general recurrent shapes,
 * gdn_short_conv_fwd, gdn_gated_rmsnorm_fwd; 1.10: gdn_chunk_bwd_workspace_bytes_for). */
int gdn_abi_version(void);

/*
 * The GPU architecture the library's kernels were compiled for, as the CUDA
 * runtime reports it for one of them (major * 10 + minor: 100 for sm_100a), or
 * -1 when no device can be queried.  Diagnostics only; no counterpart in the
 * reference.
 */
int gdn_binary_version(void);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_H */
