"""Reference-interface mirror of the FastWAM experts, backed by libfam.

The module trees below have the reference's constructor signatures,
parameter names, shapes and construction order
(FastWAM/src/fastwam/models/wan22/wan_video_dit.py:146-267 and
action_dit.py:44-100), so ``state_dict()`` / ``load_state_dict()`` are
drop-in compatible with reference checkpoints and a seeded construction draws
the same random initial weights.  torch holds the parameters and the device
buffers; every forward computation runs in libfam.so kernels through the C
ABI of include/fam.h.  There is no torch fallback: a missing library raises.

Weights are packed for the kernels (q/k/v concatenated, cross k/v
concatenated, bf16, contiguous) on first use and again after every
``load_state_dict`` (a post-hook drops the packed copy), mirroring the
reference's own post-load weight packing in its optimized trees.
"""
from __future__ import annotations

import ctypes as C
import math
from typing import List, Optional, Sequence

import torch
import torch.nn as nn

from . import _abi
from ._lib import check, lib


# ----------------------------------------------------------- module mirrors
class RMSNorm(nn.Module):
    """wan_video_dit.py:146-157 (parameter layout only)."""

    def __init__(self, dim, eps=1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))


class _Attention(nn.Module):
    def __init__(self, hidden_dim: int, attn_head_dim: int, num_heads: int, eps: float = 1e-6):
        super().__init__()
        self.hidden_dim = hidden_dim
        self.num_heads = num_heads
        self.attn_head_dim = attn_head_dim
        self.attn_hidden_dim = num_heads * attn_head_dim
        self.q = nn.Linear(hidden_dim, self.attn_hidden_dim)
        self.k = nn.Linear(hidden_dim, self.attn_hidden_dim)
        self.v = nn.Linear(hidden_dim, self.attn_hidden_dim)
        self.o = nn.Linear(self.attn_hidden_dim, hidden_dim)
        self.norm_q = RMSNorm(self.attn_hidden_dim, eps=eps)
        self.norm_k = RMSNorm(self.attn_hidden_dim, eps=eps)


class SelfAttention(_Attention):
    """wan_video_dit.py:170-195."""


class CrossAttention(_Attention):
    """wan_video_dit.py:197-219."""


class GateModule(nn.Module):
    def forward(self, x, gate, residual):  # pragma: no cover - layout only
        raise RuntimeError("GateModule runs inside libfam kernels")


class DiTBlock(nn.Module):
    """wan_video_dit.py:229-246 (same submodules, same construction order)."""

    def __init__(self, hidden_dim: int, attn_head_dim: int, num_heads: int, ffn_dim: int,
                 eps: float = 1e-6):
        super().__init__()
        self.hidden_dim = hidden_dim
        self.attn_head_dim = attn_head_dim
        self.num_heads = num_heads
        self.ffn_dim = ffn_dim
        self.self_attn = SelfAttention(hidden_dim, attn_head_dim, num_heads, eps)
        self.cross_attn = CrossAttention(hidden_dim, attn_head_dim, num_heads, eps)
        self.norm1 = nn.LayerNorm(hidden_dim, eps=eps, elementwise_affine=False)
        self.norm2 = nn.LayerNorm(hidden_dim, eps=eps, elementwise_affine=False)
        self.norm3 = nn.LayerNorm(hidden_dim, eps=eps)
        self.ffn = nn.Sequential(nn.Linear(hidden_dim, ffn_dim), nn.GELU(approximate="tanh"),
                                 nn.Linear(ffn_dim, hidden_dim))
        self.modulation = nn.Parameter(torch.randn(1, 6, hidden_dim) / hidden_dim ** 0.5)
        self.gate = GateModule()


def rope_table(head_dim: int, positions: int = 1024, theta: float = 10000.0) -> torch.Tensor:
    """(cos, sin) of precompute_freqs_cis(head_dim) (wan_video_dit.py:45-51): angles in fp64,
    stored fp32 [positions, head_dim/2, 2]."""
    freqs = 1.0 / (theta ** (torch.arange(0, head_dim, 2)[: head_dim // 2].double() / head_dim))
    ang = torch.outer(torch.arange(positions, dtype=torch.float64), freqs)
    return torch.stack([ang.cos(), ang.sin()], dim=-1).float().contiguous()


class ActionDiT(nn.Module):
    """Action expert (action_dit.py:44-100): same constructor and state_dict."""

    def __init__(self, hidden_dim: int, action_dim: int, ffn_dim: int, text_dim: int,
                 freq_dim: int, eps: float, num_heads: int, attn_head_dim: int, num_layers: int,
                 use_gradient_checkpointing: bool = False):
        super().__init__()
        self.hidden_dim = hidden_dim
        self.action_dim = action_dim
        self.ffn_dim = ffn_dim
        self.text_dim = text_dim
        self.freq_dim = freq_dim
        self.num_heads = num_heads
        self.attn_head_dim = attn_head_dim
        self.eps = eps
        if num_heads <= 0 or attn_head_dim <= 0 or attn_head_dim % 2:
            raise ValueError("num_heads > 0 and an even attn_head_dim are required")
        self.action_encoder = nn.Linear(action_dim, hidden_dim)
        self.text_embedding = nn.Sequential(nn.Linear(text_dim, hidden_dim),
                                            nn.GELU(approximate="tanh"),
                                            nn.Linear(hidden_dim, hidden_dim))
        self.time_embedding = nn.Sequential(nn.Linear(freq_dim, hidden_dim), nn.SiLU(),
                                            nn.Linear(hidden_dim, hidden_dim))
        self.time_projection = nn.Sequential(nn.SiLU(), nn.Linear(hidden_dim, hidden_dim * 6))
        self.blocks = nn.ModuleList([DiTBlock(hidden_dim, attn_head_dim, num_heads, ffn_dim, eps)
                                     for _ in range(num_layers)])
        self.head = nn.Linear(hidden_dim, action_dim)
        self.use_gradient_checkpointing = use_gradient_checkpointing
        self._engine: Optional["ActionExpertEngine"] = None
        self.register_load_state_dict_post_hook(lambda module, keys: module._invalidate())

    def _invalidate(self):
        self._engine = None

    def _apply(self, fn, *args, **kwargs):
        self._engine = None
        return super()._apply(fn, *args, **kwargs)

    @property
    def num_layers(self) -> int:
        return len(self.blocks)

    def engine(self) -> "ActionExpertEngine":
        if self._engine is None:
            self._engine = ActionExpertEngine(self)
        return self._engine

    def forward(self, action_tokens, timestep, context, context_mask=None):
        """ActionDiT.forward (action_dit.py:333-362): the expert alone, no video cache."""
        return self.engine().denoise_step(action_tokens, timestep, context, context_mask)


# ------------------------------------------------------------------ engine
class ActionExpertEngine:
    """Owns the packed weights, the libfam handle and the workspace of one expert."""

    def __init__(self, dit: ActionDiT):
        p = next(dit.parameters())
        if not p.is_cuda:
            raise RuntimeError("ActionDiT must be on a CUDA device for the libfam path")
        self.dev = p.device
        self.dit = dit
        bfw = lambda t: t.detach().to(device=self.dev, dtype=torch.bfloat16).contiguous()
        self.keep: List[torch.Tensor] = []

        def ptr(t):
            self.keep.append(t)
            return t.data_ptr()

        layers = (_abi.ActionLayer * dit.num_layers)()
        for i, b in enumerate(dit.blocks):
            sa, ca = b.self_attn, b.cross_attn
            L = layers[i]
            L.modulation = ptr(bfw(b.modulation.reshape(6, -1)))
            L.qkv_w = ptr(bfw(torch.cat([sa.q.weight, sa.k.weight, sa.v.weight], 0)))
            L.qkv_b = ptr(bfw(torch.cat([sa.q.bias, sa.k.bias, sa.v.bias], 0)))
            L.norm_q, L.norm_k = ptr(bfw(sa.norm_q.weight)), ptr(bfw(sa.norm_k.weight))
            L.o_w, L.o_b = ptr(bfw(sa.o.weight)), ptr(bfw(sa.o.bias))
            L.norm3_w, L.norm3_b = ptr(bfw(b.norm3.weight)), ptr(bfw(b.norm3.bias))
            L.cq_w, L.cq_b = ptr(bfw(ca.q.weight)), ptr(bfw(ca.q.bias))
            L.cnorm_q, L.cnorm_k = ptr(bfw(ca.norm_q.weight)), ptr(bfw(ca.norm_k.weight))
            L.ckv_w = ptr(bfw(torch.cat([ca.k.weight, ca.v.weight], 0)))
            L.ckv_b = ptr(bfw(torch.cat([ca.k.bias, ca.v.bias], 0)))
            L.co_w, L.co_b = ptr(bfw(ca.o.weight)), ptr(bfw(ca.o.bias))
            L.ffn0_w, L.ffn0_b = ptr(bfw(b.ffn[0].weight)), ptr(bfw(b.ffn[0].bias))
            L.ffn2_w, L.ffn2_b = ptr(bfw(b.ffn[2].weight)), ptr(bfw(b.ffn[2].bias))
        w = _abi.ActionWeights()
        for name, mod in (("enc", dit.action_encoder), ("text0", dit.text_embedding[0]),
                          ("text2", dit.text_embedding[2]), ("time0", dit.time_embedding[0]),
                          ("time2", dit.time_embedding[2]), ("tproj", dit.time_projection[1]),
                          ("head", dit.head)):
            setattr(w, name + "_w", ptr(bfw(mod.weight)))
            setattr(w, name + "_b", ptr(bfw(mod.bias)))
        self._layers = layers
        w.layers = layers
        w.rope = ptr(rope_table(dit.attn_head_dim).to(self.dev))
        w.rope_positions = 1024
        cfg = _abi.ActionConfig(dit.hidden_dim, dit.action_dim, dit.ffn_dim, dit.text_dim,
                                dit.freq_dim, dit.num_heads, dit.attn_head_dim, dit.num_layers,
                                float(dit.eps))
        self._weights = w
        h = C.c_void_p()
        with torch.cuda.device(self.dev):
            check(lib().fam_action_expert_create(C.byref(cfg), C.byref(w), C.byref(h)),
                  "fam_action_expert_create")
        self.handle = h
        self.ws: Optional[torch.Tensor] = None

    def __del__(self):
        h = getattr(self, "handle", None)
        if h is not None and h.value:
            try:
                lib().fam_action_expert_destroy(h)
            except Exception:
                pass

    def _workspace(self, B, Sa, C_, N) -> torch.Tensor:
        n = C.c_size_t()
        check(lib().fam_action_workspace_size(self.handle, B, Sa, C_, N, C.byref(n)),
              "fam_action_workspace_size")
        if self.ws is None or self.ws.numel() < n.value:
            self.ws = torch.empty(n.value, dtype=torch.uint8, device=self.dev)
        return self.ws

    def _io(self, B, Sa, context, context_mask, cache_k, cache_v, attn_mask, N):
        io = _abi.ActionIO()
        io.batch, io.action_tokens = B, Sa
        ctx = context.to(device=self.dev, dtype=torch.bfloat16).contiguous()
        self._ctx = ctx
        io.context_tokens = ctx.shape[1]
        io.context = ctx.data_ptr()
        if context_mask is not None:
            cm = context_mask.to(device=self.dev, dtype=torch.uint8)
            cm = cm.expand(B, ctx.shape[1]).contiguous() if cm.dim() == 2 else cm
            self._cm = cm
            io.context_mask = cm.data_ptr()
        if cache_k is not None and len(cache_k) > 0:
            ks = [k if k.dtype == torch.bfloat16 else k.bfloat16() for k in cache_k]
            vs = [v if v.dtype == torch.bfloat16 else v.bfloat16() for v in cache_v]
            k0 = ks[0]
            if k0.stride(-1) != 1 or any(k.stride() != k0.stride() for k in ks + vs):
                raise ValueError("video K/V caches must share one strided layout with unit last stride")
            io.video_tokens = k0.shape[1]
            io.video_batch_stride, io.video_token_stride = k0.stride(0), k0.stride(1)
            self._kp = (C.c_void_p * len(ks))(*[k.data_ptr() for k in ks])
            self._vp = (C.c_void_p * len(vs))(*[v.data_ptr() for v in vs])
            self._kv_keep = (ks, vs)
            io.video_k = C.cast(self._kp, C.POINTER(C.c_void_p))
            io.video_v = C.cast(self._vp, C.POINTER(C.c_void_p))
        if attn_mask is not None:
            am = attn_mask.to(device=self.dev, dtype=torch.uint8).contiguous()
            self._am = am
            io.attn_mask = am.data_ptr()
        ws = self._workspace(B, Sa, io.context_tokens, N)
        io.workspace, io.workspace_bytes = ws.data_ptr(), ws.numel()
        return io

    def launch_count(self) -> int:
        """Kernels the last chunk / step call enqueued (a graph replay launches the same)."""
        n = C.c_int32()
        check(lib().fam_action_launch_count(self.handle, C.byref(n)), "fam_action_launch_count")
        return n.value

    def denoise_step(self, latents, timestep, context, context_mask=None, cache_k=None,
                     cache_v=None, attn_mask=None) -> torch.Tensor:
        """One model evaluation (FastWAM._denoise_action_with_video_cache, fastwam.py:771-804)."""
        lat = latents.to(device=self.dev, dtype=torch.bfloat16).contiguous()
        B, Sa, _ = lat.shape
        io = self._io(B, Sa, context, context_mask, cache_k, cache_v, attn_mask, 1)
        vel = torch.empty_like(lat)
        t = float(timestep.reshape(-1)[0].item()) if torch.is_tensor(timestep) else float(timestep)
        st = torch.cuda.current_stream(self.dev).cuda_stream
        check(lib().fam_action_denoise_step(self.handle, C.byref(io), lat.data_ptr(), t,
                                            vel.data_ptr(), C.c_void_p(st)),
              "fam_action_denoise_step")
        return vel

    def chunk(self, latents, timesteps: Sequence[float], deltas: Sequence[float], context,
              context_mask=None, cache_k=None, cache_v=None, attn_mask=None,
              return_trace: bool = False, use_graph: bool = True, out: Optional[torch.Tensor] = None):
        """The Euler loop of FastWAM.infer_action (fastwam.py:1241-1263); latent updated in place
        in `out` (a bf16 copy of `latents` when not given)."""
        lat = out if out is not None else latents.to(device=self.dev, dtype=torch.bfloat16).clone()
        B, Sa, A = lat.shape
        N = len(timesteps)
        io = self._io(B, Sa, context, context_mask, cache_k, cache_v, attn_mask, N)
        trace = torch.empty((N, B, Sa, A), dtype=torch.bfloat16, device=self.dev) if return_trace else None
        ts = (C.c_float * N)(*[float(t) for t in timesteps])
        ds = (C.c_float * N)(*[float(d) for d in deltas])
        st = torch.cuda.current_stream(self.dev).cuda_stream
        check(lib().fam_action_chunk(self.handle, C.byref(io), lat.data_ptr(), ts, ds, N,
                                     trace.data_ptr() if trace is not None else None,
                                     1 if use_graph else 0, C.c_void_p(st)), "fam_action_chunk")
        return (lat, trace) if return_trace else lat


# ---------------------------------------------------------------- schedule
def build_inference_schedule(num_inference_steps: int, shift: float, dtype=torch.bfloat16,
                             num_train_timesteps: int = 1000):
    """WanContinuousFlowMatchScheduler.build_inference_schedule (scheduler_continuous.py:63-80),
    host-side: the (dtype-rounded) timesteps and deltas handed to the chunk kernels."""
    if num_inference_steps <= 0 or shift <= 0:
        raise ValueError("num_inference_steps and shift must be positive")
    u = torch.linspace(1.0, 0.0, num_inference_steps + 1, dtype=torch.float32)
    sigma = shift * u / (1.0 + (shift - 1.0) * u)
    t = (sigma[:-1] * float(num_train_timesteps)).to(dtype)
    d = (sigma[1:] - sigma[:-1]).to(dtype)
    return t.float().tolist(), d.float().tolist()
