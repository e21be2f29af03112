"""``GatedDeltaNetModel`` in PyTorch, with the delta-rule layer on this library's kernels.

Mirrors the reference's Flax modules (``src/gated_deltanet_jax/model.py``): the
class names, constructor arguments (a :class:`GatedDeltaNetConfig`), parameter
names and the forward computation are the reference's, so a caller that builds
the model from a config and feeds token ids gets the same network:

* ``GatedDeltaNet`` (model.py:58-156): q/k/v/a/b(/g) projections, the short
  convolutions with SiLU (model.py:15-40, :119-122; or SiLU alone without them),
  grouped value heads without repeating q/k (model.py:132-135), the gates
  ``beta = sigmoid(b)``, ``g = -exp(A_log) softplus(a + dt_bias)`` (:136-139),
  the mode switch (:141-146), the gated RMSNorm (:147-153) and ``o_proj``;
* ``GatedDeltaNetMLP`` (:162-180), ``GatedDeltaNetBlock`` (:186-205),
  ``GatedDeltaNetModel`` (:211-230), ``GatedDeltaNetForCausalLM`` (:236-245).

The GatedDeltaNet-specific work runs on the CUDA kernels: the short convolution
(``ops.short_convolution``), and the gates + delta rule + gated RMSNorm in one
call (``ops.gated_delta_rule_chunk_layer`` in ``'chunk'`` mode on its tensor-core
shapes, ``ops.gated_delta_rule_decode_layer`` in ``'fused_recurrent'`` mode; the
separate ops elsewhere).  Embedding, RMSNorm, projections and the MLP are plain
torch operations (cuBLAS GEMMs).  The fused forms have no backward: when
gradients are wanted, the layer takes the differentiable route instead (torch
short convolution and gated RMSNorm, the delta rule through the ops' autograd,
whose backward is ``gdn_chunk_bwd``).

Like the reference, the layer applies no L2 norm and no 1/sqrt(dk) scale to q
and k, so at the default initialisation the recurrence grows by orders of
magnitude per token and long sequences overflow (in the reference as well).

Weights use torch's layout (``nn.Linear``: ``[out, in]``; the reference's Flax
kernels are ``[in, out]``); the short-convolution weights are ``[K, C]`` (the
Flax depthwise kernel ``[K, 1, C]`` squeezed).
"""

from __future__ import annotations

import math
from typing import Optional

import torch
from torch import nn
import torch.nn.functional as F

from . import dispatch, ops
from .configuration import GatedDeltaNetConfig

__all__ = ["ShortConvolution", "GatedDeltaNet", "GatedDeltaNetMLP", "GatedDeltaNetBlock",
           "GatedDeltaNetModel", "GatedDeltaNetForCausalLM", "RMSNorm"]


def _lecun_normal_(w: torch.Tensor, fan_in: int) -> torch.Tensor:
    # the Flax default kernel initialiser (variance 1 / fan_in, truncated normal
    # approximated by a normal here)
    with torch.no_grad():
        return w.normal_(0.0, 1.0 / math.sqrt(fan_in))


def _linear(d_in: int, d_out: int) -> nn.Linear:
    lin = nn.Linear(d_in, d_out, bias=False)
    _lecun_normal_(lin.weight, d_in)
    return lin


class ShortConvolution(nn.Module):
    """Causal depthwise convolution over time, kernel K, then SiLU (model.py:15-40).
    ``weight`` [K, C] (the Flax depthwise kernel [K, 1, C] squeezed), optional bias.
    On the GPU kernel (gdn_short_conv_fwd) for inference; torch's conv1d when
    gradients are wanted or with a bias."""

    def __init__(self, hidden_size: int, kernel_size: int, activation: Optional[str] = "silu",
                 use_bias: bool = False):
        super().__init__()
        self.hidden_size, self.kernel_size, self.activation = hidden_size, kernel_size, activation
        # Flax's fan-in for a depthwise kernel is K
        self.weight = nn.Parameter(_lecun_normal_(torch.empty(kernel_size, hidden_size),
                                                  kernel_size))
        self.bias = nn.Parameter(torch.zeros(hidden_size)) if use_bias else None

    def forward(self, x):
        act = self.activation in ("silu", "swish")
        grad = torch.is_grad_enabled() and (
            x.requires_grad or any(p.requires_grad for p in self.parameters()))
        if not grad and self.bias is None:
            y, _ = ops.short_convolution(x.contiguous(), self.weight.detach().float(),
                                         activation="silu" if act else None)
            return y
        K, C = self.weight.shape
        xt = F.pad(x.transpose(1, 2), (K - 1, 0))
        bias = None if self.bias is None else self.bias.to(x.dtype)
        y = F.conv1d(xt, self.weight.t().reshape(C, 1, K).to(x.dtype), bias, groups=C)
        y = y.transpose(1, 2)
        return F.silu(y) if act else y


class RMSNorm(nn.Module):
    """``x rsqrt(mean(x^2) + eps) scale`` over the last dimension (Flax
    ``nnx.RMSNorm``), the statistic in fp32."""

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        if x.is_cuda and hasattr(F, "rms_norm"):   # one fused pass (fp32 accumulation)
            return F.rms_norm(x, (x.shape[-1],), self.weight.to(x.dtype), self.eps)
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight.float()
        return y.to(x.dtype)


class GatedDeltaNet(nn.Module):
    """The GatedDeltaNet attention layer (model.py:58-156)."""

    def __init__(self, config: GatedDeltaNetConfig, layer_idx: Optional[int] = None):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.hidden_size = config.hidden_size
        self.num_heads = config.num_heads
        self.num_v_heads = config.num_v_heads if config.num_v_heads is not None else config.num_heads
        self.head_k_dim = config.head_dim
        self.head_v_dim = int(config.head_dim * config.expand_v)
        self.key_dim = self.num_heads * self.head_k_dim
        self.value_dim = self.num_v_heads * self.head_v_dim
        if self.num_v_heads % self.num_heads:
            raise ValueError("num_v_heads must be a multiple of num_heads")
        D = config.hidden_size
        self.q_proj = _linear(D, self.key_dim)
        self.k_proj = _linear(D, self.key_dim)
        self.v_proj = _linear(D, self.value_dim)
        self.a_proj = _linear(D, self.num_v_heads)
        self.b_proj = _linear(D, self.num_v_heads)
        self.g_proj = _linear(D, self.value_dim) if config.use_gate else None
        # FusedRMSNormGated (eps 1e-5) with a gate; nnx.RMSNorm (eps 1e-6) without
        self.o_norm_weight = nn.Parameter(torch.ones(self.head_v_dim))
        self.o_norm_eps = 1e-5 if config.use_gate else 1e-6
        self.o_proj = _linear(self.value_dim, D)
        if config.use_short_conv:
            K = config.conv_size
            self.q_conv = ShortConvolution(self.key_dim, K)
            self.k_conv = ShortConvolution(self.key_dim, K)
            self.v_conv = ShortConvolution(self.value_dim, K)
        # A in U(1e-4, 16); dt log-uniform in [1e-3, 0.1], dt_bias its inverse softplus
        A = torch.empty(self.num_v_heads).uniform_(1e-4, 16.0)
        self.A_log = nn.Parameter(torch.log(A))
        dt = torch.exp(torch.empty(self.num_v_heads).uniform_(math.log(1e-3), math.log(0.1)))
        dt = dt.clamp_min(1e-4)
        self.dt_bias = nn.Parameter(dt + torch.log(-torch.expm1(-dt)))

    def _fused_shape(self, dtype) -> bool:
        return (dtype == torch.bfloat16 and self.head_k_dim in (128, 256)
                and self.head_v_dim % 64 == 0)

    def forward(self, x, mask=None):
        B, T, _ = x.shape
        grad = torch.is_grad_enabled() and (
            x.requires_grad or any(p.requires_grad for p in self.parameters()))
        q, k, v = self.q_proj(x), self.k_proj(x), self.v_proj(x)
        if self.config.use_short_conv:
            q, k, v = self.q_conv(q), self.k_conv(k), self.v_conv(v)
        else:
            q, k, v = F.silu(q), F.silu(k), F.silu(v)
        # grouped value heads: q/k keep num_heads heads (the kernels read head
        # h * num_heads / num_v_heads), no repeat
        q = q.reshape(B, T, self.num_heads, self.head_k_dim)
        k = k.reshape(B, T, self.num_heads, self.head_k_dim)
        v = v.reshape(B, T, self.num_v_heads, self.head_v_dim)
        a = self.a_proj(x).float()
        b = self.b_proj(x).float()
        gate = None
        if self.g_proj is not None:
            gate = self.g_proj(x).reshape(B, T, self.num_v_heads, self.head_v_dim)
        mode = self.config.attn_mode
        if mode not in ("chunk", "fused_recurrent"):
            raise ValueError(f"Unknown mode {mode}")
        A_log, dt_bias, w = self.A_log, self.dt_bias, self.o_norm_weight
        if not grad and mode == "chunk" and self._fused_shape(q.dtype):
            o, _ = ops.gated_delta_rule_chunk_layer(q, k, v, a, b, A_log, dt_bias, gate=gate,
                                                    norm_weight=w, eps=self.o_norm_eps)
        elif not grad and mode == "fused_recurrent":
            o, _ = ops.gated_delta_rule_decode_layer(q, k, v, a, b, A_log, dt_bias, gate=gate,
                                                     norm_weight=w, eps=self.o_norm_eps)
        else:
            # the separate operations (model.py:136-153)
            beta = torch.sigmoid(b)
            g = -torch.exp(A_log.float()) * F.softplus(a + dt_bias.float())
            o = dispatch.delta_rule(self.config, q, k, v, g, beta)
            if grad:
                of = o.float()
                y = of * torch.rsqrt(of.pow(2).mean(-1, keepdim=True) + self.o_norm_eps)
                y = y * w.float()
                if gate is not None:
                    y = y * F.silu(gate.float())
                o = y.to(v.dtype)
            else:
                o = ops.gated_rms_norm(o, gate, w.float(), self.o_norm_eps)
        return self.o_proj(o.reshape(B, T, self.value_dim))


class GatedDeltaNetMLP(nn.Module):
    """SwiGLU MLP (model.py:162-180)."""

    def __init__(self, config: GatedDeltaNetConfig):
        super().__init__()
        self.hidden_size = config.hidden_size
        inter = config.intermediate_size
        if inter is None:
            inter = int(config.hidden_size * config.hidden_ratio * 2 / 3)
            inter = 256 * ((inter + 256 - 1) // 256)
        self.intermediate_size = inter
        self.gate_proj = _linear(config.hidden_size, inter)
        self.up_proj = _linear(config.hidden_size, inter)
        self.down_proj = _linear(inter, config.hidden_size)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class GatedDeltaNetBlock(nn.Module):
    """Pre-norm residual block: attention, then MLP (model.py:186-205)."""

    def __init__(self, config: GatedDeltaNetConfig, layer_idx: int):
        super().__init__()
        self.attn_norm = RMSNorm(config.hidden_size, eps=config.norm_eps)
        self.attn = GatedDeltaNet(config, layer_idx=layer_idx)
        self.mlp_norm = RMSNorm(config.hidden_size, eps=config.norm_eps)
        self.mlp = GatedDeltaNetMLP(config)

    def forward(self, x, mask=None):
        x = x + self.attn(self.attn_norm(x), mask=mask)
        return x + self.mlp(self.mlp_norm(x))


class GatedDeltaNetModel(nn.Module):
    """Embedding, ``num_hidden_layers`` blocks, final RMSNorm (model.py:211-230)."""

    def __init__(self, config: GatedDeltaNetConfig):
        super().__init__()
        self.config = config
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size)
        with torch.no_grad():   # Flax's Embed default: variance 1 / features
            self.embed_tokens.weight.normal_(0.0, 1.0 / math.sqrt(config.hidden_size))
        self.layers = nn.ModuleList(GatedDeltaNetBlock(config, layer_idx=i)
                                    for i in range(config.num_hidden_layers))
        self.norm = RMSNorm(config.hidden_size, eps=config.norm_eps)

    def forward(self, input_ids):
        x = self.embed_tokens(input_ids)
        for layer in self.layers:
            x = layer(x, mask=None)
        return self.norm(x)


class GatedDeltaNetForCausalLM(nn.Module):
    """The model plus its LM head (model.py:236-245)."""

    def __init__(self, config: GatedDeltaNetConfig):
        super().__init__()
        self.config = config
        self.model = GatedDeltaNetModel(config)
        self.lm_head = _linear(config.hidden_size, config.vocab_size)

    def forward(self, input_ids):
        return self.lm_head(self.model(input_ids))
