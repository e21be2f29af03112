// Single-token decode step with the state streamed through shared memory by
// bulk (TMA) copies, sm_100a.
//
// Same math as recurrent.cu (the reference recurrence, ops.py:170-184), for
// T == 1 and heads whose fp32 state fits one shared-memory stage
// (dk * dv * 4 <= 64 KB).  A head's state [dk, dv] is one contiguous block, so
// each head moves with one cp.async.bulk load and one cp.async.bulk store:
//
//   * persistent grid: one CTA per SM, heads assigned round-robin;
//   * a producer warp keeps NS stages in flight: it waits until the compute
//     warps have released a stage, bulk-stores the updated state from it,
//     and bulk-loads the state (plus the head's q, k, v) of a later head;
//   * 8 compute warps: each thread holds 4 columns x RPT rows of the state in
//     registers, reduces k^T S and q^T S (warp shuffles, then an mbarrier-
//     synchronised exchange between warps), writes o, updates the state and
//     writes it back into the stage for the producer to store.
//
// HBM traffic per head: the state read and written once, plus q, k, v, o,
// g, beta.  Every mbarrier wait is bounded (ptx.cuh).
//
// The layer form (kLayer) also does the work of the GatedDeltaNet layer on
// either side of the step (model.py:136-139 and :47-53), for one token:
//   prologue  beta = sigmoid(b), g = -exp(A_log[h]) softplus(a + dt_bias[h]),
//             from the raw a_proj / b_proj outputs a, b;
//   epilogue  y = o rsqrt(mean(o^2) + eps) w (silu(gate) if a gate is given),
//             over the head's dv outputs, which warp 0 holds (4 per lane), in
//             fp32 before the one rounding to the output dtype.
#include <cstdlib>

#include "gdn_common.cuh"
#include "gdn_internal.h"
#include "ptx.cuh"

namespace gdn {

namespace {

constexpr int kStages = 3;
constexpr int kComputeWarps = 8;
constexpr int kComputeThreads = kComputeWarps * 32;
constexpr int kThreads = kComputeThreads + 32;  // + producer warp

template <typename Tin, int DK, int DV>
struct BulkLayout {
  static constexpr int LPR = DV / 4;
  static constexpr int state_bytes = DK * DV * 4;
  static constexpr int qk_bytes = DK * (int)sizeof(Tin);
  static constexpr int v_bytes = DV * (int)sizeof(Tin);
  static constexpr int stage_bytes = state_bytes + 2 * qk_bytes + v_bytes;
  static constexpr int red_bytes = 2 * kComputeWarps * 2 * LPR * 16;  // double buffered
  static constexpr int total = kStages * stage_bytes + red_bytes;
  static_assert(state_bytes % 16 == 0 && qk_bytes % 16 == 0 && v_bytes % 16 == 0, "bulk sizes");
};

// Four consecutive input elements kept as loaded (no conversion yet), so that
// a load issued ahead of its use does not wait for its data where it is issued.
template <typename Tin> struct Raw4;
template <> struct Raw4<float> {
  float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
  __device__ void load(const float* p) { r = *reinterpret_cast<const float4*>(p); }
  __device__ float4 get() const { return r; }
};
template <> struct Raw4<__nv_bfloat16> {
  uint2 r = make_uint2(0u, 0u);
  __device__ void load(const __nv_bfloat16* p) { r = *reinterpret_cast<const uint2*>(p); }
  __device__ float4 get() const {
    return make_float4(__uint_as_float(r.x << 16), __uint_as_float(r.x & 0xffff0000u),
                       __uint_as_float(r.y << 16), __uint_as_float(r.y & 0xffff0000u));
  }
};

template <typename Tin, int DK, int DV, bool kLayer>
__global__ void __launch_bounds__(kThreads, 1)
recurrent_bulk_kernel(const Tin* __restrict__ q, const Tin* __restrict__ k,
                      const Tin* __restrict__ v, const float* __restrict__ g,
                      const float* __restrict__ beta, const float* h0, Tin* __restrict__ o,
                      float* hT, int n_units, int H, int Hk, const LayerArgs la) {
  using L = BulkLayout<Tin, DK, DV>;
  constexpr int LPR = L::LPR;
  constexpr int RPP = kComputeThreads / LPR;
  constexpr int RPT = DK / RPP;
  static_assert(LPR <= 32 && 32 % LPR == 0 && DK % RPP == 0 && RPT >= 1, "tile");
  static_assert(!kLayer || LPR == 32, "the layer epilogue needs a head's outputs in one warp");

  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint64_t full_bar[kStages], free_bar[kStages], red_bar[2];

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int my_units = n_units > (int)blockIdx.x
                           ? (n_units - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&free_bar[s], kComputeWarps);
    }
    mbar_init(&red_bar[0], kComputeWarps);
    mbar_init(&red_bar[1], kComputeWarps);
    fence_mbar_init();
  }
  __syncthreads();
  // Everything above overlaps the previous decode step; nothing in global
  // memory is read before that step has completed.
  griddep_wait();
  if (tid == 0) griddep_launch_dependents();

  auto stage = [&](int s) { return smem + (size_t)s * L::stage_bytes; };

  if (warp == kComputeWarps) {
    // ---------------- producer warp ----------------
    if (!elect_one()) return;
    auto unit_of = [&](int j) { return (int)blockIdx.x + j * (int)gridDim.x; };
    auto load = [&](int j) {
      const int s = j % kStages, u = unit_of(j);
      // q/k row of this (b, h): value head h reads q/k head h * Hk / H (grouped heads)
      const int uq = (u / H) * Hk + (u % H) * Hk / H;
      unsigned char* st = stage(s);
      const uint32_t bytes = (h0 ? L::state_bytes : 0) + 2 * L::qk_bytes + L::v_bytes;
      mbar_arrive_expect_tx(&full_bar[s], bytes);
      if (h0) bulk_g2s(st, h0 + (size_t)u * DK * DV, L::state_bytes, &full_bar[s]);
      bulk_g2s(st + L::state_bytes, q + (size_t)uq * DK, L::qk_bytes, &full_bar[s]);
      bulk_g2s(st + L::state_bytes + L::qk_bytes, k + (size_t)uq * DK, L::qk_bytes, &full_bar[s]);
      bulk_g2s(st + L::state_bytes + 2 * L::qk_bytes, v + (size_t)u * DV, L::v_bytes,
               &full_bar[s]);
    };
    auto release = [&](int j) -> bool {  // store the state of unit j once computed
      const int s = j % kStages;
      if (!mbar_wait(&free_bar[s], (uint32_t)(j / kStages) & 1u)) return false;
      if (hT) {
        bulk_s2g(hT + (size_t)unit_of(j) * DK * DV, stage(s), L::state_bytes);
        bulk_commit();
      }
      return true;
    };
    int issued = 0;
    bool ok = true;
    for (int j = 0; j < my_units && ok; ++j) {
      if (j >= kStages) {
        ok = release(j - kStages);
        if (!ok) break;
        bulk_wait_read<0>();  // the stage may be overwritten once the store has read it
      }
      load(j);
      issued = j + 1;
    }
    for (int j = my_units > kStages ? my_units - kStages : 0; ok && j < my_units; ++j)
      ok = release(j);
    if (!ok) {  // a wait gave up: let the loads still in flight land before exiting
      for (int j = issued > kStages ? issued - kStages : 0; j < issued; ++j)
        mbar_wait(&full_bar[j % kStages], (uint32_t)(j / kStages) & 1u);
    }
    bulk_wait<0>();
    return;
  }

  // ---------------- compute warps ----------------
  float4* red = reinterpret_cast<float4*>(smem + (size_t)kStages * L::stage_bytes);
  const int cg = tid % LPR, rb = tid / LPR;
  const int unit0 = blockIdx.x;
  // (layer form: g_next / b_next hold the raw a / b, gate_next the output gate)
  float g_next = 0.f, b_next = 0.f;
  Raw4<Tin> gate_next;
  float4 w4 = make_float4(0.f, 0.f, 0.f, 0.f);
  const Tin* gate = static_cast<const Tin*>(la.gate);
  if (kLayer && rb == 0) w4 = *reinterpret_cast<const float4*>(la.weight + cg * 4);
  // layer form: model.py:136-139 from the raw a, b and the head's A_log, dt_bias
  auto layer_gates = [&](float a_raw, float b_raw, float A, float dtb, float& gg, float& bb) {
    gg = -expf(A) * softplus(a_raw + dtb);
    bb = sigmoid(b_raw);
  };
  float g_cur = 0.f, b_cur = 0.f;   // layer form: the current unit's g and beta
  float A_next = 0.f, dtb_next = 0.f;
  if (my_units > 0) {
    g_next = kLayer ? la.a[unit0] : g[unit0];
    b_next = kLayer ? la.b[unit0] : beta[unit0];
    if (kLayer) {
      A_next = la.A_log[unit0 % H];
      dtb_next = la.dt_bias[unit0 % H];
      if (gate && rb == 0) gate_next.load(gate + (size_t)unit0 * DV + cg * 4);
      layer_gates(g_next, b_next, A_next, dtb_next, g_cur, b_cur);
    }
  }
  for (int j = 0; j < my_units; ++j) {
    const int s = j % kStages, u = unit0 + j * (int)gridDim.x;
    // layer form, warp 0: norm weight x silu(gate) of this unit, computed before
    // the unit's state arrives (the gate was fetched with the previous unit)
    float4 gw = w4;
    if (kLayer && gate && rb == 0) {
      const float4 gv = gate_next.get();
      gw.x *= gv.x * sigmoid(gv.x); gw.y *= gv.y * sigmoid(gv.y);
      gw.z *= gv.z * sigmoid(gv.z); gw.w *= gv.w * sigmoid(gv.w);
    }
    // (layer form: the gates were computed at the end of the previous unit, off
    // this unit's critical path)
    const float alpha = __expf(kLayer ? g_cur : g_next), bt = kLayer ? b_cur : b_next;
    if (j + 1 < my_units) {  // prefetch the next head's gate and beta
      const int un = u + (int)gridDim.x;
      g_next = kLayer ? la.a[un] : g[un];
      b_next = kLayer ? la.b[un] : beta[un];
      if (kLayer) {
        A_next = la.A_log[un % H];
        dtb_next = la.dt_bias[un % H];
        if (gate && rb == 0) gate_next.load(gate + (size_t)un * DV + cg * 4);
      }
    }
    if (!mbar_wait(&full_bar[s], (uint32_t)(j / kStages) & 1u)) return;
    unsigned char* st = stage(s);
    float* Ss = reinterpret_cast<float*>(st);
    const Tin* qs = reinterpret_cast<const Tin*>(st + L::state_bytes);
    const Tin* ks = reinterpret_cast<const Tin*>(st + L::state_bytes + L::qk_bytes);
    const Tin* vs = reinterpret_cast<const Tin*>(st + L::state_bytes + 2 * L::qk_bytes);

    float4 S[RPT];
    float4 kh = make_float4(0.f, 0.f, 0.f, 0.f), qh = kh;
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const int r = rb + i * RPP;
      S[i] = h0 ? *reinterpret_cast<const float4*>(Ss + r * DV + cg * 4)
                : make_float4(0.f, 0.f, 0.f, 0.f);
      const float kr = to_f32(ks[r]), qr = to_f32(qs[r]);
      kh = fma4(kr, S[i], kh);
      qh = fma4(qr, S[i], qh);
    }
    // q . k, reduced within every warp (each warp needs it).
    float qk = 0.f;
#pragma unroll
    for (int d = lane; d < DK; d += 32) qk = fmaf(to_f32(qs[d]), to_f32(ks[d]), qk);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) qk += __shfl_xor_sync(0xffffffffu, qk, off);
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
    }
    float4* rbuf = red + (size_t)(j & 1) * kComputeWarps * 2 * LPR;
    if (lane < LPR) {
      rbuf[(warp * 2 + 0) * LPR + lane] = kh;
      rbuf[(warp * 2 + 1) * LPR + lane] = qh;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&red_bar[j & 1]);
    if (!mbar_wait(&red_bar[j & 1], (uint32_t)(j >> 1) & 1u)) return;
    kh = rbuf[cg];
    qh = rbuf[LPR + cg];
#pragma unroll
    for (int w = 1; w < kComputeWarps; ++w) {
      const float4 a = rbuf[(w * 2 + 0) * LPR + cg], c = rbuf[(w * 2 + 1) * LPR + cg];
      kh.x += a.x; kh.y += a.y; kh.z += a.z; kh.w += a.w;
      qh.x += c.x; qh.y += c.y; qh.z += c.z; qh.w += c.w;
    }
    const float4 vv = load4(vs + cg * 4);
    float4 uu;
    uu.x = bt * (vv.x - alpha * kh.x);
    uu.y = bt * (vv.y - alpha * kh.y);
    uu.z = bt * (vv.z - alpha * kh.z);
    uu.w = bt * (vv.w - alpha * kh.w);
    if (rb == 0) {
      float4 out;
      out.x = fmaf(alpha, qh.x, qk * uu.x);
      out.y = fmaf(alpha, qh.y, qk * uu.y);
      out.z = fmaf(alpha, qh.z, qk * uu.z);
      out.w = fmaf(alpha, qh.w, qk * uu.w);
      if (kLayer) {   // model.py:47-53, over the head's DV outputs held by this warp
        float ss = out.x * out.x + out.y * out.y + out.z * out.z + out.w * out.w;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        const float rs = rsqrtf(ss * (1.f / DV) + la.eps);
        out.x *= rs * gw.x; out.y *= rs * gw.y; out.z *= rs * gw.z; out.w *= rs * gw.w;
      }
      store4(o + (size_t)u * DV + cg * 4, out);
    }
    if (hT) {
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        const int r = rb + i * RPP;
        const float kr = to_f32(ks[r]);
        float4 n;
        n.x = fmaf(alpha, S[i].x, kr * uu.x);
        n.y = fmaf(alpha, S[i].y, kr * uu.y);
        n.z = fmaf(alpha, S[i].z, kr * uu.z);
        n.w = fmaf(alpha, S[i].w, kr * uu.w);
        *reinterpret_cast<float4*>(Ss + r * DV + cg * 4) = n;
      }
      fence_proxy_async_smem();
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&free_bar[s]);
    if (kLayer && j + 1 < my_units) layer_gates(g_next, b_next, A_next, dtb_next, g_cur, b_cur);
  }
}

int num_sms() { return device_sm_count(); }

template <typename Tin, int DK, int DV, bool kLayer>
cudaError_t launch_bulk_t(const RecurrentArgs& a, const LayerArgs& la, cudaStream_t st) {
  using L = BulkLayout<Tin, DK, DV>;
  auto kern = recurrent_bulk_kernel<Tin, DK, DV, kLayer>;
  static std::atomic<int> smem_set[kMaxDevices] = {};
  cudaError_t e = ensure_smem(kern, L::total, smem_set);
  if (e != cudaSuccess) return e;
  const int n_units = a.B * a.H;
  const int grid = n_units < num_sms() ? n_units : num_sms();
  // Consecutive decode steps on one stream may overlap their launch and
  // set-up (programmatic dependent launch); GDN_DECODE_PDL=0 turns it off.
  const bool pdl = kernel_overrides().decode_pdl;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L::total;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, static_cast<const Tin*>(a.q), static_cast<const Tin*>(a.k),
                         static_cast<const Tin*>(a.v), a.g, a.beta, a.h0, static_cast<Tin*>(a.o),
                         a.hT, n_units, a.H, a.Hk, la);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace

GDN_DEVICE_ERROR_ACCESSOR(device_error_recurrent_bulk)

bool recurrent_bulk_supported(const RecurrentArgs& a) {
  return a.T == 1 && a.dk == 128 && a.dv == 128;
}

cudaError_t launch_recurrent_bulk(const RecurrentArgs& a, cudaStream_t st) {
  if (a.B * a.H == 0) return cudaSuccess;
  const LayerArgs none{};
  return a.dtype == kBF16 ? launch_bulk_t<__nv_bfloat16, 128, 128, false>(a, none, st)
                          : launch_bulk_t<float, 128, 128, false>(a, none, st);
}

cudaError_t launch_recurrent_bulk_layer(const RecurrentArgs& a, const LayerArgs& la,
                                        cudaStream_t st) {
  if (a.B * a.H == 0) return cudaSuccess;
  return a.dtype == kBF16 ? launch_bulk_t<__nv_bfloat16, 128, 128, true>(a, la, st)
                          : launch_bulk_t<float, 128, 128, true>(a, la, st);
}

}  // namespace gdn
