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

from . import _abi, ops
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


class PreparedVideo:
    """The token stage of WanVideoDiT.prepare (wan_video_dit.py:640-720) as this library
    runs it: patch embedding, the per-token time MLPs and the text embedding are fused
    into the prefill kernels, so prepare() hands the prefill its inputs (the latent grid,
    per-sample timesteps, the raw context) in this record.  It stands in the reference's
    `tokens` / `t` / `t_mod` slots; `.shape` is the token tensor's [B, S, D]."""

    def __init__(self, latents, timestep, context, context_mask, grid, hidden_dim):
        self.latents, self.timestep = latents, timestep
        self.context, self.context_mask = context, context_mask
        self.grid = grid
        self.shape = torch.Size((latents.shape[0], grid[0] * grid[1] * grid[2], hidden_dim))


class PreparedAction:
    """The token stage of ActionDiT.prepare (action_dit.py:312-327): the action encoder,
    the time MLP and the text embedding run inside the action-expert kernels, so
    prepare() hands them the noisy latents, the timestep (a host value) and the raw
    context.  `.shape` is the token tensor's [B, Sa, D]."""

    def __init__(self, latents, timestep, context, context_mask, hidden_dim):
        self.latents, self.timestep = latents, timestep
        self.context, self.context_mask = context, context_mask
        self.shape = torch.Size((latents.shape[0], latents.shape[1], hidden_dim))


class ActionStepOut:
    """MoT.forward_action_with_video_cache_tensor's output as this library runs it: the
    step kernels end with the head (ActionDiT.post), so the record carries the velocity."""

    def __init__(self, velocity):
        self.velocity = velocity
        self.shape = velocity.shape


def _host_timestep(timestep):
    """A timestep as host floats (a tensor on the GPU is read back once)."""
    if torch.is_tensor(timestep):
        return [float(x) for x in timestep.reshape(-1).float().tolist()]
    if isinstance(timestep, (list, tuple)):
        return [float(x) for x in timestep]
    return [float(timestep)]


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

    def is_compact(self) -> bool:
        """Hidden <= 64 experts (the CAE expert) run the persistent fp32 kernel."""
        return (self.hidden_dim <= 64 and self.num_heads * self.attn_head_dim <= 64
                and self.attn_head_dim <= 32 and self.ffn_dim <= 256)

    def engine(self):
        """ActionExpertEngine (bf16 tcgen05 path) or CAEEngine (compact experts)."""
        if self._engine is None:
            self._engine = CAEEngine(self) if self.is_compact() else ActionExpertEngine(self)
        return self._engine

    def forward(self, action_tokens, timestep, context, context_mask=None):
        """ActionDiT.forward (action_dit.py:333-362): the expert alone, no video cache."""
        return self.engine().denoise_step(action_tokens, timestep, context, context_mask)

    def prepare(self, action_tokens, timestep, context, context_mask=None):
        """ActionDiT.prepare (action_dit.py:312-327) -> (tokens, t, t_mod, context,
        context_mask, freqs) in the reference's order; tokens / t / t_mod are one
        PreparedAction record (the stage runs inside the step kernels) and freqs the RoPE
        table of the action positions."""
        prep = PreparedAction(action_tokens, _host_timestep(timestep)[0], context, context_mask,
                              self.hidden_dim)
        freqs = rope_table(self.attn_head_dim, action_tokens.shape[1])
        return prep, prep, prep, context, context_mask, freqs

    def post(self, x):
        """ActionDiT.post (action_dit.py:329-331): the head, already applied by the step
        kernels; returns the velocity of an ActionStepOut."""
        if not isinstance(x, ActionStepOut):
            raise TypeError("ActionDiT.post takes the output of MoT.forward_action_with_video_cache_tensor")
        return x.velocity


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

        # Every per-block tensor is packed into one contiguous stack over the blocks
        # (block i at rows i * N): the launch chain uses per-block slices, the fused
        # persistent kernel streams whole stacks through single tensor maps.
        blocks = list(dit.blocks)

        def stack(fn):
            t = torch.stack([fn(b).detach().to(device=self.dev, dtype=torch.bfloat16)
                             for b in blocks]).contiguous()
            self.keep.append(t)
            return t

        S = {
            "modulation": stack(lambda b: b.modulation.reshape(6, -1)),
            "qkv_w": stack(lambda b: torch.cat([b.self_attn.q.weight, b.self_attn.k.weight,
                                                b.self_attn.v.weight], 0)),
            "qkv_b": stack(lambda b: torch.cat([b.self_attn.q.bias, b.self_attn.k.bias,
                                                b.self_attn.v.bias], 0)),
            "norm_q": stack(lambda b: b.self_attn.norm_q.weight),
            "norm_k": stack(lambda b: b.self_attn.norm_k.weight),
            "o_w": stack(lambda b: b.self_attn.o.weight), "o_b": stack(lambda b: b.self_attn.o.bias),
            "norm3_w": stack(lambda b: b.norm3.weight), "norm3_b": stack(lambda b: b.norm3.bias),
            "cq_w": stack(lambda b: b.cross_attn.q.weight), "cq_b": stack(lambda b: b.cross_attn.q.bias),
            "cnorm_q": stack(lambda b: b.cross_attn.norm_q.weight),
            "cnorm_k": stack(lambda b: b.cross_attn.norm_k.weight),
            "ckv_w": stack(lambda b: torch.cat([b.cross_attn.k.weight, b.cross_attn.v.weight], 0)),
            "ckv_b": stack(lambda b: torch.cat([b.cross_attn.k.bias, b.cross_attn.v.bias], 0)),
            "co_w": stack(lambda b: b.cross_attn.o.weight), "co_b": stack(lambda b: b.cross_attn.o.bias),
            "ffn0_w": stack(lambda b: b.ffn[0].weight), "ffn0_b": stack(lambda b: b.ffn[0].bias),
            "ffn2_w": stack(lambda b: b.ffn[2].weight), "ffn2_b": stack(lambda b: b.ffn[2].bias),
        }
        layers = (_abi.ActionLayer * dit.num_layers)()
        for i in range(dit.num_layers):
            for name, t in S.items():
                setattr(layers[i], name, t[i].data_ptr())
        stacks = _abi.ActionStacks()
        for name, _ in _abi.ActionStacks._fields_:
            setattr(stacks, name, S[name].data_ptr())
        self._stacks = stacks
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
        w.stacks = C.pointer(stacks)
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

    MODES = {"auto": 0, "chain": 1, "fused": 2}

    def set_mode(self, mode: str) -> None:
        """'auto' (fused persistent kernel when the call qualifies), 'chain' or 'fused'."""
        check(lib().fam_action_set_mode(self.handle, self.MODES[mode]), "fam_action_set_mode")

    def last_path(self) -> str:
        n = C.c_int32()
        check(lib().fam_action_last_path(self.handle, C.byref(n)), "fam_action_last_path")
        return {0: "none", 1: "chain", 2: "fused"}[n.value]

    def set_kernel_events(self, start=None, stop=None) -> None:
        """Record two torch.cuda.Event objects around the fused kernel of every
        fused-path chunk called with use_graph=False (None, None clears).  The
        events must have been recorded once (torch creates the CUDA event lazily)."""
        hs = C.c_void_p(start.cuda_event) if start is not None else None
        he = C.c_void_p(stop.cuda_event) if stop is not None else None
        check(lib().fam_action_set_kernel_events(self.handle, hs, he), "fam_action_set_kernel_events")

    def denoise_step(self, latents, timestep, context, context_mask=None, cache_k=None,
                     cache_v=None, attn_mask=None) -> torch.Tensor:
        """One model evaluation (FastWAM._denoise_action_with_video_cache, fastwam.py:771-804).
        timestep: a float, or a one-value tensor; the kernels take it as a launch argument,
        so a tensor on the GPU costs a device-to-host read (a stream synchronisation) that a
        host value does not."""
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


# ------------------------------------------------------------ video DiT
class Head(nn.Module):
    """wan_video_dit.py:287-306 (parameter layout)."""

    def __init__(self, dim: int, out_dim: int, patch_size, eps: float):
        super().__init__()
        self.dim = dim
        self.patch_size = patch_size
        self.norm = nn.LayerNorm(dim, eps=eps, elementwise_affine=False)
        self.head = nn.Linear(dim, out_dim * math.prod(patch_size))
        self.modulation = nn.Parameter(torch.randn(1, 2, dim) / dim ** 0.5)


def rope_table_3d(head_dim: int, f: int, h: int, w: int, theta: float = 10000.0) -> torch.Tensor:
    """Per-token (cos, sin) of WanVideoDiT.get_freqs (wan_video_dit.py:37-51, 406-415): the
    head is split (d - 2(d//3), d//3, d//3) over (frame, row, column); angles in fp64,
    stored fp32 [f*h*w, d/2, 2]."""
    def freqs(dim):
        return 1.0 / (theta ** (torch.arange(0, dim, 2)[: dim // 2].double() / dim))
    df = head_dim - 2 * (head_dim // 3)
    dh = head_dim // 3
    ff, fh, fw = freqs(df), freqs(dh), freqs(dh)
    fi = torch.arange(f, dtype=torch.float64).view(f, 1, 1, 1).expand(f, h, w, 1)
    hi = torch.arange(h, dtype=torch.float64).view(1, h, 1, 1).expand(f, h, w, 1)
    wi = torch.arange(w, dtype=torch.float64).view(1, 1, w, 1).expand(f, h, w, 1)
    ang = torch.cat([fi * ff, hi * fh, wi * fw], dim=-1).reshape(f * h * w, -1)
    return torch.stack([ang.cos(), ang.sin()], dim=-1).float().contiguous()


class WanVideoDiT(nn.Module):
    """Video expert (wan_video_dit.py:308-405): same constructor signature, parameters and
    construction order.  prefill() runs WanVideoDiT.prepare + MoT.prefill_video_cache_tensor
    through fam_video_prefill."""

    def __init__(self, hidden_dim: int, in_dim: int, ffn_dim: int, out_dim: int, text_dim: int,
                 freq_dim: int, eps: float, patch_size, num_heads: int, attn_head_dim: int,
                 num_layers: int, has_image_input: bool, has_image_pos_emb: bool = False,
                 has_ref_conv: bool = False, add_control_adapter: bool = False,
                 in_dim_control_adapter: int = 24, seperated_timestep: bool = False,
                 require_vae_embedding: bool = False, require_clip_embedding: bool = False,
                 fuse_vae_embedding_in_latents: bool = True, action_conditioned: bool = False,
                 action_dim: int = 7, action_group_causal_mask_mode="causal",
                 video_attention_mask_mode: str = "bidirectional",
                 use_gradient_checkpointing: bool = False):
        super().__init__()
        if has_image_input or require_clip_embedding or require_vae_embedding:
            raise ValueError("image input / clip / vae embeddings are not supported (as in the reference)")
        if attn_head_dim % 2:
            raise ValueError("attn_head_dim must be even for RoPE")
        self.hidden_dim, self.in_dim, self.freq_dim = hidden_dim, in_dim, freq_dim
        self.patch_size = tuple(patch_size)
        self.num_heads, self.attn_head_dim, self.eps = num_heads, attn_head_dim, eps
        self.ffn_dim, self.text_dim = ffn_dim, text_dim
        self.seperated_timestep = seperated_timestep
        self.fuse_vae_embedding_in_latents = fuse_vae_embedding_in_latents
        self.video_attention_mask_mode = str(video_attention_mask_mode)
        self.action_conditioned = action_conditioned
        self.action_dim = action_dim
        self.patch_embedding = nn.Conv3d(in_dim, hidden_dim, kernel_size=patch_size, stride=patch_size)
        self.text_embedding = nn.Sequential(nn.Linear(text_dim, hidden_dim), nn.GELU(approximate="tanh"),
                                            nn.Linear(hidden_dim, hidden_dim))
        self.time_embedding = nn.Sequential(nn.Linear(freq_dim, hidden_dim), nn.SiLU(),
                                            nn.Linear(hidden_dim, hidden_dim))
        self.time_projection = nn.Sequential(nn.SiLU(), nn.Linear(hidden_dim, hidden_dim * 6))
        self.blocks = nn.ModuleList([DiTBlock(hidden_dim, attn_head_dim, num_heads, ffn_dim, eps)
                                     for _ in range(num_layers)])
        self.head = Head(hidden_dim, out_dim, patch_size, eps)
        if has_ref_conv:
            self.ref_conv = nn.Conv2d(16, hidden_dim, kernel_size=(2, 2), stride=(2, 2))
        if action_conditioned:
            self.action_embedding = nn.Linear(action_dim, hidden_dim)
        self.use_gradient_checkpointing = use_gradient_checkpointing
        self._engine = None
        self.register_load_state_dict_post_hook(lambda m, k: setattr(m, "_engine", None))

    def _apply(self, fn, *args, **kwargs):
        self._engine = None
        return super()._apply(fn, *args, **kwargs)

    @property
    def num_layers(self) -> int:
        return len(self.blocks)

    def engine(self) -> "VideoPrefillEngine":
        if self._engine is None:
            self._engine = VideoPrefillEngine(self)
        return self._engine

    def prefill(self, latents, timestep, context, context_mask=None, return_hidden=False):
        return self.engine().prefill(latents, timestep, context, context_mask, return_hidden)

    def prepare(self, x, timestep, context, context_mask=None, action=None, fuse_vae_embedding_in_latents=True):
        """WanVideoDiT.prepare (wan_video_dit.py:640-720) -> (tokens, t, t_mod, context,
        context_mask, freqs, f, h, w, tokens_per_frame) in the reference's order; tokens /
        t / t_mod are one PreparedVideo record (patch embedding, time MLPs and text
        embedding run inside the prefill kernels), freqs the 3-D RoPE table."""
        if action is not None:
            raise ValueError("action-conditioned prepare is not on this path")
        if not fuse_vae_embedding_in_latents:
            raise ValueError("only fuse_vae_embedding_in_latents=True exists (as in the reference)")
        pt, ph, pw = self.patch_size
        f, h, w = x.shape[2] // pt, x.shape[3] // ph, x.shape[4] // pw
        prep = PreparedVideo(x, _host_timestep(timestep), context, context_mask, (f, h, w), self.hidden_dim)
        freqs = rope_table_3d(self.attn_head_dim, f, h, w)
        return prep, prep, prep, context, context_mask, freqs, f, h, w, h * w

    def build_video_to_video_mask(self, video_seq_len: int, video_tokens_per_frame: int, device=None):
        """WanVideoDiT.build_video_to_video_mask (wan_video_dit.py:489-523), bool."""
        mode = self.video_attention_mask_mode
        if mode == "bidirectional":
            return torch.ones((video_seq_len, video_seq_len), dtype=torch.bool, device=device)
        if mode == "first_frame_causal":
            m = torch.ones((video_seq_len, video_seq_len), dtype=torch.bool, device=device)
            ff = min(video_tokens_per_frame, video_seq_len)
            m[:ff, ff:] = False
            return m
        if mode == "per_frame_causal":
            nf = video_seq_len // video_tokens_per_frame
            fc = torch.tril(torch.ones((nf, nf), dtype=torch.bool, device=device))
            return fc.repeat_interleave(video_tokens_per_frame, 0).repeat_interleave(video_tokens_per_frame, 1)
        raise ValueError(f"unknown video_attention_mask_mode {mode!r}")


class VideoPrefillEngine:
    """Packed bf16 weights + fam_video_expert handle + workspace of one WanVideoDiT."""

    def __init__(self, dit: WanVideoDiT, stack_cross_kv: bool = True):
        """stack_cross_kv: store every block's cross K/V projection in one block-major
        allocation (one context GEMM per prefill); False keeps one allocation per block
        (one GEMM per block, the same result)."""
        p = next(dit.parameters())
        if not p.is_cuda:
            raise RuntimeError("WanVideoDiT must be on a CUDA device for the libfam path")
        if not (dit.seperated_timestep and dit.fuse_vae_embedding_in_latents):
            raise ValueError("only the separated-timestep, fused-VAE-latent path exists (as in the reference)")
        self.dev = p.device
        self.dit = dit
        self.keep: List[torch.Tensor] = []
        self._head = None
        bfw = lambda t: t.detach().to(device=self.dev, dtype=torch.bfloat16).contiguous()

        def ptr(t):
            self.keep.append(t)
            return t.data_ptr()

        layers = (_abi.ActionLayer * dit.num_layers)()
        # every block's cross K/V projection and norm_k stacked block-major, so the
        # prefill projects the (step-invariant) context for all blocks in one GEMM
        ckv_w = bfw(torch.stack([torch.cat([b.cross_attn.k.weight, b.cross_attn.v.weight], 0) for b in dit.blocks]))
        ckv_b = bfw(torch.stack([torch.cat([b.cross_attn.k.bias, b.cross_attn.v.bias], 0) for b in dit.blocks]))
        cnorm_k = bfw(torch.stack([b.cross_attn.norm_k.weight for b in dit.blocks]))
        self.keep += [ckv_w, ckv_b, cnorm_k]
        for i, b in enumerate(dit.blocks):
            sa, ca, L = b.self_attn, b.cross_attn, layers[i]
            L.modulation = ptr(bfw(b.modulation.reshape(6, -1)))
            L.qkv_w = ptr(bfw(torch.cat([sa.q.weight, sa.k.weight, sa.v.weight], 0)))
            L.qkv_b = ptr(bfw(torch.cat([sa.q.bias, sa.k.bias, sa.v.bias], 0)))
            L.norm_q, L.norm_k = ptr(bfw(sa.norm_q.weight)), ptr(bfw(sa.norm_k.weight))
            L.o_w, L.o_b = ptr(bfw(sa.o.weight)), ptr(bfw(sa.o.bias))
            L.norm3_w, L.norm3_b = ptr(bfw(b.norm3.weight)), ptr(bfw(b.norm3.bias))
            L.cq_w, L.cq_b = ptr(bfw(ca.q.weight)), ptr(bfw(ca.q.bias))
            if stack_cross_kv:
                L.cnorm_k, L.ckv_w, L.ckv_b = cnorm_k[i].data_ptr(), ckv_w[i].data_ptr(), ckv_b[i].data_ptr()
            else:
                L.cnorm_k, L.ckv_w, L.ckv_b = (ptr(cnorm_k[i].clone()), ptr(ckv_w[i].clone()),
                                               ptr(ckv_b[i].clone()))
            L.cnorm_q = ptr(bfw(ca.norm_q.weight))
            L.co_w, L.co_b = ptr(bfw(ca.o.weight)), ptr(bfw(ca.o.bias))
            L.ffn0_w, L.ffn0_b = ptr(bfw(b.ffn[0].weight)), ptr(bfw(b.ffn[0].bias))
            L.ffn2_w, L.ffn2_b = ptr(bfw(b.ffn[2].weight)), ptr(bfw(b.ffn[2].bias))
        w = _abi.VideoWeights()
        w.patch_w = ptr(bfw(dit.patch_embedding.weight.reshape(dit.hidden_dim, -1)))
        w.patch_b = ptr(bfw(dit.patch_embedding.bias))
        for name, mod in (("text0", dit.text_embedding[0]), ("text2", dit.text_embedding[2]),
                          ("time0", dit.time_embedding[0]), ("time2", dit.time_embedding[2]),
                          ("tproj", dit.time_projection[1])):
            setattr(w, name + "_w", ptr(bfw(mod.weight)))
            setattr(w, name + "_b", ptr(bfw(mod.bias)))
        self._layers = layers
        w.layers = layers
        pt, ph, pw = dit.patch_size
        cfg = _abi.VideoConfig(dit.hidden_dim, dit.in_dim, dit.ffn_dim, dit.text_dim, dit.freq_dim,
                               dit.num_heads, dit.attn_head_dim, dit.num_layers, pt, ph, pw,
                               float(dit.eps))
        self._w = w
        h = C.c_void_p()
        with torch.cuda.device(self.dev):
            check(lib().fam_video_expert_create(C.byref(cfg), C.byref(w), C.byref(h)),
                  "fam_video_expert_create")
        self.handle = h
        self.ws: Optional[torch.Tensor] = None
        self._rope = {}
        self.last = None

    def __del__(self):
        h = getattr(self, "handle", None)
        if h is not None and h.value:
            try:
                lib().fam_video_expert_destroy(h)
            except Exception:
                pass

    def launch_count(self) -> int:
        n = C.c_int32()
        check(lib().fam_video_launch_count(self.handle, C.byref(n)), "fam_video_launch_count")
        return n.value

    def rope(self, f, h, w) -> torch.Tensor:
        key = (f, h, w)
        if key not in self._rope:
            self._rope[key] = rope_table_3d(self.dit.attn_head_dim, f, h, w).to(self.dev)
        return self._rope[key]

    def prefill(self, latents, timestep, context, context_mask=None, return_hidden=False,
                cache_k=None, cache_v=None, hidden=None, use_graph=True, t_out=None):
        """WanVideoDiT.prepare + MoT.prefill_video_cache_tensor: returns the per-block K and V
        lists ([B, S, H*d] bf16) and, with return_hidden, the final token states (fp32).
        timestep: a float, a list of floats (one per sample) or a tensor; the kernels take the
        values as launch arguments, so a tensor on the GPU costs a device-to-host read.
        t_out (bf16 [B, 2, D], optional) receives the time embedding rows for post()."""
        d = self.dit
        lat = latents.to(device=self.dev, dtype=torch.bfloat16).contiguous()
        B, _, Fr, Hh, Ww = lat.shape
        pt, ph, pw = d.patch_size
        f, hh, ww = Fr // pt, Hh // ph, Ww // pw
        S = f * hh * ww
        HD = d.num_heads * d.attn_head_dim
        if cache_k is None:
            cache_k = [torch.empty(B, S, HD, dtype=torch.bfloat16, device=self.dev) for _ in range(d.num_layers)]
            cache_v = [torch.empty(B, S, HD, dtype=torch.bfloat16, device=self.dev) for _ in range(d.num_layers)]
        if return_hidden and hidden is None:
            hidden = torch.empty(B, S, d.hidden_dim, dtype=torch.float32, device=self.dev)
        ctx = context.to(device=self.dev, dtype=torch.bfloat16).contiguous()
        Cc = ctx.shape[1]
        cm = None
        if context_mask is not None:
            cm = context_mask.to(device=self.dev, dtype=torch.uint8).expand(B, Cc).contiguous()
        if torch.is_tensor(timestep):
            tsv = timestep.reshape(-1).float().tolist()
        elif isinstance(timestep, (list, tuple)):
            tsv = [float(x) for x in timestep]
        else:
            tsv = [float(timestep)]
        if len(tsv) == 1:
            tsv = tsv * B
        io = _abi.VideoIO()
        io.batch, io.frames, io.height, io.width, io.context_tokens = B, Fr, Hh, Ww, Cc
        io.latents = lat.data_ptr()
        ts = (C.c_float * B)(*tsv)
        io.timesteps = ts
        io.context = ctx.data_ptr()
        io.context_mask = cm.data_ptr() if cm is not None else None
        rope = self.rope(f, hh, ww)
        io.rope = rope.data_ptr()
        io.first_frame_causal = 1 if d.video_attention_mask_mode == "first_frame_causal" else 0
        if d.video_attention_mask_mode not in ("first_frame_causal", "bidirectional"):
            raise ValueError("video_attention_mask_mode must be first_frame_causal or bidirectional")
        kp = (C.c_void_p * d.num_layers)(*[k.data_ptr() for k in cache_k])
        vpp = (C.c_void_p * d.num_layers)(*[v.data_ptr() for v in cache_v])
        io.cache_k = C.cast(kp, C.POINTER(C.c_void_p))
        io.cache_v = C.cast(vpp, C.POINTER(C.c_void_p))
        io.hidden_out = hidden.data_ptr() if hidden is not None else None
        io.t_out = t_out.data_ptr() if t_out is not None else None
        n = C.c_size_t()
        check(lib().fam_video_workspace_size(self.handle, B, S, Cc, C.byref(n)), "fam_video_workspace_size")
        if self.ws is None or self.ws.numel() < n.value:
            self.ws = torch.empty(n.value, dtype=torch.uint8, device=self.dev)
        io.workspace, io.workspace_bytes = self.ws.data_ptr(), self.ws.numel()
        st = torch.cuda.current_stream(self.dev).cuda_stream
        check(lib().fam_video_prefill(self.handle, C.byref(io), 1 if use_graph else 0, C.c_void_p(st)),
              "fam_video_prefill")
        self.last = (lat, ctx, cm, rope, kp, vpp, ts)  # keep inputs alive until the work is done
        return (cache_k, cache_v, hidden) if return_hidden else (cache_k, cache_v)

    def post(self, hidden, t_rows, grid, first_frame_tokens, out=None):
        """WanVideoDiT.post_dit (wan_video_dit.py:634-638): Head.forward with the per-token
        time embedding, then unpatchify -> bf16 [B, out_dim, F, H, W].  hidden: fp32
        [B, S, D] from prefill(return_hidden=True); t_rows: its t_out."""
        d = self.dit
        B, S, D = hidden.shape
        f, h, w = grid
        pt, ph, pw = d.patch_size
        hw = d.head
        if self._head is None:
            self._head = (hw.head.weight.detach().to(self.dev, torch.bfloat16).contiguous(),
                          hw.head.bias.detach().to(self.dev, torch.bfloat16).contiguous(),
                          hw.modulation.detach().reshape(2, D).to(self.dev, torch.bfloat16).contiguous())
        wgt, bias, mod = self._head
        st = C.c_void_p(torch.cuda.current_stream(self.dev).cuda_stream)
        normed = torch.empty(B * S, D, dtype=torch.bfloat16, device=self.dev)
        check(lib().fam_video_head_norm(C.c_void_p(hidden.data_ptr()), C.c_void_p(t_rows.data_ptr()),
                                        C.c_void_p(mod.data_ptr()), B, S, first_frame_tokens, D, float(d.eps),
                                        C.c_void_p(normed.data_ptr()), st), "fam_video_head_norm")
        proj = ops.gemm(normed, wgt, bias=bias)
        Cout = wgt.shape[0] // (pt * ph * pw)
        if out is None:
            out = torch.empty(B, Cout, f * pt, h * ph, w * pw, dtype=torch.bfloat16, device=self.dev)
        check(lib().fam_video_unpatchify(C.c_void_p(proj.data_ptr()), B, f, h, w, pt, ph, pw, Cout,
                                         C.c_void_p(out.data_ptr()), st), "fam_video_unpatchify")
        self.last_post = (normed, proj)
        return out


# ---------------------------------------------------- compact expert engine
def _f32(t: torch.Tensor, dev) -> torch.Tensor:
    return t.detach().to(device=dev, dtype=torch.float32).contiguous()


class CAEEngine:
    """Compact action expert (hidden <= 64): fp32 weights, the whole Euler loop of a
    chunk in two launches (fam_cae_chunk)."""

    def __init__(self, dit: "ActionDiT"):
        p = next(dit.parameters())
        if not p.is_cuda:
            raise RuntimeError("ActionDiT must be on a CUDA device for the libfam path")
        self.dev = p.device
        self.dit = dit
        self.keep: List[torch.Tensor] = []

        def ptr(t):
            t = _f32(t, self.dev)
            self.keep.append(t)
            return t.data_ptr()

        layers = (_abi.CaeLayer * dit.num_layers)()
        for i, b in enumerate(dit.blocks):
            sa, ca, L = b.self_attn, b.cross_attn, layers[i]
            L.modulation = ptr(b.modulation.reshape(6, -1))
            L.qkv_w = ptr(torch.cat([sa.q.weight, sa.k.weight, sa.v.weight], 0))
            L.qkv_b = ptr(torch.cat([sa.q.bias, sa.k.bias, sa.v.bias], 0))
            L.norm_q, L.norm_k = ptr(sa.norm_q.weight), ptr(sa.norm_k.weight)
            L.o_w, L.o_b = ptr(sa.o.weight), ptr(sa.o.bias)
            L.norm3_w, L.norm3_b = ptr(b.norm3.weight), ptr(b.norm3.bias)
            L.cq_w, L.cq_b = ptr(ca.q.weight), ptr(ca.q.bias)
            L.cnorm_q, L.cnorm_k = ptr(ca.norm_q.weight), ptr(ca.norm_k.weight)
            L.ckv_w = ptr(torch.cat([ca.k.weight, ca.v.weight], 0))
            L.ckv_b = ptr(torch.cat([ca.k.bias, ca.v.bias], 0))
            L.co_w, L.co_b = ptr(ca.o.weight), ptr(ca.o.bias)
            L.ffn0_w, L.ffn0_b = ptr(b.ffn[0].weight), ptr(b.ffn[0].bias)
            L.ffn2_w, L.ffn2_b = ptr(b.ffn[2].weight), ptr(b.ffn[2].bias)
        w = _abi.CaeWeights()
        for name, mod in (("enc", dit.action_encoder), ("text0", dit.text_embedding[0]),
                          ("text2", dit.text_embedding[2]), ("time0", dit.time_embedding[0]),
                          ("time2", dit.time_embedding[2]), ("tproj", dit.time_projection[1]),
                          ("head", dit.head)):
            setattr(w, name + "_w", ptr(mod.weight))
            setattr(w, name + "_b", ptr(mod.bias))
        self._layers = layers
        w.layers = layers
        w.rope = ptr(rope_table(dit.attn_head_dim))
        w.rope_positions = 1024
        self._w = w
        self.cfg = _abi.ActionConfig(dit.hidden_dim, dit.action_dim, dit.ffn_dim, dit.text_dim,
                                     dit.freq_dim, dit.num_heads, dit.attn_head_dim,
                                     dit.num_layers, float(dit.eps))
        self.ws: Optional[torch.Tensor] = None

    def chunk(self, latents, timesteps: Sequence[float], deltas: Sequence[float], context,
              context_mask=None, return_trace: bool = False, out: Optional[torch.Tensor] = None):
        """Euler loop over ActionDiT.forward (action_dit.py:333-362) -> fp32 latent [B,S,A]."""
        lat = out if out is not None else latents.to(device=self.dev, dtype=torch.float32).clone()
        B, S, A = lat.shape
        ctx = context if context.is_cuda and context.dtype in (torch.bfloat16, torch.float32) \
            else context.to(self.dev, torch.float32)
        ctx = ctx.contiguous()
        C_ = ctx.shape[1]
        cm = None
        if context_mask is not None:
            cm = context_mask.to(device=self.dev, dtype=torch.uint8).expand(B, C_).contiguous()
        n = C.c_size_t()
        check(lib().fam_cae_workspace_size(C.byref(self.cfg), B, C_, C.byref(n)), "fam_cae_workspace_size")
        if self.ws is None or self.ws.numel() < n.value:
            self.ws = torch.empty(n.value, dtype=torch.uint8, device=self.dev)
        N = len(timesteps)
        trace = torch.empty((N, B, S, A), dtype=torch.float32, device=self.dev) if return_trace else None
        ts = (C.c_float * N)(*[float(t) for t in timesteps])
        ds = (C.c_float * N)(*[float(d) for d in deltas])
        st = torch.cuda.current_stream(self.dev).cuda_stream
        check(lib().fam_cae_chunk(C.byref(self.cfg), C.byref(self._w), B, S, ctx.data_ptr(),
                                  1 if ctx.dtype == torch.bfloat16 else 0, C_,
                                  cm.data_ptr() if cm is not None else None, lat.data_ptr(), ts, ds,
                                  N, trace.data_ptr() if trace is not None else None,
                                  self.ws.data_ptr(), self.ws.numel(), C.c_void_p(st)),
              "fam_cae_chunk")
        self._hold = (ctx, cm)
        self._last = (B, C_)
        return (lat, trace) if return_trace else lat

    DECODE_MODES = {"auto": 0, "fused": 1, "separate": 2}

    def chunk_decode(self, latents, timesteps: Sequence[float], deltas: Sequence[float], context, ae: "ActionAE",
                     context_mask=None, suite_ids=None, decode: str = "auto"):
        """The Euler loop and ActionAE.decode of the final latents (fam_cae_chunk_decode).  The
        decode can run in the step kernel's epilogue when the decoder qualifies (one upsampling
        stage of stride 2 or 4); decode="auto" takes it at batch >= 4 (where it beats the
        separate launches), "fused" whenever it qualifies, "separate" never.
        Returns (fp32 latents [B, S, A], fp32 actions [B, horizon, action_dim]);
        self.decode_fused tells which way the decode ran."""
        if decode not in self.DECODE_MODES:
            raise ValueError(f"decode must be one of {sorted(self.DECODE_MODES)}")
        lat = latents.to(device=self.dev, dtype=torch.float32).clone()
        B, S, A = lat.shape
        ctx = context if context.is_cuda and context.dtype in (torch.bfloat16, torch.float32) \
            else context.to(self.dev, torch.float32)
        ctx = ctx.contiguous()
        C_ = ctx.shape[1]
        cm = None
        if context_mask is not None:
            cm = context_mask.to(device=self.dev, dtype=torch.uint8).expand(B, C_).contiguous()
        dec = ae.decoder
        dec.check_ids(suite_ids)
        if dec._packed is None:
            dec._pack()
        dcfg, dw, _, _ = dec._packed
        n = C.c_size_t()
        check(lib().fam_cae_decode_workspace_size(C.byref(self.cfg), C.byref(dcfg), C.byref(dw), B, C_,
                                                  C.byref(n)), "fam_cae_decode_workspace_size")
        if self.ws is None or self.ws.numel() < n.value:
            self.ws = torch.empty(n.value, dtype=torch.uint8, device=self.dev)
        N = len(timesteps)
        ts = (C.c_float * N)(*[float(t) for t in timesteps])
        ds = (C.c_float * N)(*[float(d) for d in deltas])
        out = torch.empty((B, ae.cfg.action_horizon, ae.cfg.action_dim), dtype=torch.float32, device=self.dev)
        sid = None
        if suite_ids is not None and dec.suite_embed is not None:
            sid = suite_ids.to(device=self.dev, dtype=torch.int32).contiguous()
        fused = C.c_int32(0)
        st = torch.cuda.current_stream(self.dev).cuda_stream
        check(lib().fam_cae_chunk_decode(C.byref(self.cfg), C.byref(self._w), B, S, ctx.data_ptr(),
                                         1 if ctx.dtype == torch.bfloat16 else 0, C_,
                                         cm.data_ptr() if cm is not None else None, lat.data_ptr(), ts, ds, N,
                                         None, C.byref(dcfg), C.byref(dw),
                                         sid.data_ptr() if sid is not None else None, out.data_ptr(),
                                         self.DECODE_MODES[decode], C.byref(fused), self.ws.data_ptr(),
                                         self.ws.numel(), C.c_void_p(st)),
              "fam_cae_chunk_decode")
        self.decode_fused = bool(fused.value)
        self._hold = (ctx, cm, sid)
        self._last = (B, C_)
        return lat, out

    def status(self) -> int:
        """Status word of the last chunk (0 = every bounded device wait completed)."""
        B, C_ = self._last
        out = C.c_int32(0)
        st = torch.cuda.current_stream(self.dev).cuda_stream
        check(lib().fam_cae_status(C.byref(self.cfg), B, C_, self.ws.data_ptr(), C.byref(out), C.c_void_p(st)),
              "fam_cae_status")
        return out.value

    def denoise_step(self, latents, timestep, context, context_mask=None):
        """One model evaluation (ActionDiT.forward) -> velocity fp32 [B,S,A]."""
        t = float(timestep.reshape(-1)[0].item()) if torch.is_tensor(timestep) else float(timestep)
        _, tr = self.chunk(latents, [t], [0.0], context, context_mask, return_trace=True)
        return tr[0]


# ------------------------------------------------------------ action VAE
from dataclasses import dataclass


@dataclass
class ActionAEConfig:
    """FastWAM/src/fastwam/models/action_ae.py:16-30."""

    action_dim: int = 7
    action_horizon: int = 32
    num_tokens: int = 4
    latent_dim: int = 8
    encoder_hidden: int = 128
    decoder_hidden: int = 128
    video_cond_dim: int = 12288
    variational: bool = False
    beta_kl: float = 1e-2
    free_bits: float = 0.0
    recon_loss: str = "mse"
    num_suites: int = 0
    sigreg_lambda: float = 0.0


def _factorise_ratio(ratio: int) -> List[int]:
    """ActionEncoder._factorise_ratio (action_ae.py:95-107)."""
    if ratio == 1:
        return [1]
    out = []
    for f in (4, 2, 3):
        while ratio % f == 0:
            out.append(f)
            ratio //= f
    if ratio > 1:
        out.append(ratio)
    return out


class ResidualConv1dBlock(nn.Module):
    """action_ae.py:33-47 (layout)."""

    def __init__(self, channels: int, kernel_size: int = 3):
        super().__init__()
        pad = kernel_size // 2
        self.net = nn.Sequential(nn.Conv1d(channels, channels, kernel_size, padding=pad),
                                 nn.GroupNorm(min(8, channels), channels), nn.SiLU(),
                                 nn.Conv1d(channels, channels, kernel_size, padding=pad),
                                 nn.GroupNorm(min(8, channels), channels))


class ActionEncoder(nn.Module):
    """action_ae.py:50-121 (parameter layout; encoding is not on the denoising path)."""

    def __init__(self, cfg: ActionAEConfig):
        super().__init__()
        self.cfg = cfg
        if cfg.action_horizon % cfg.num_tokens:
            raise ValueError("action_horizon must be divisible by num_tokens")
        self.input_proj = nn.Linear(cfg.action_dim, cfg.encoder_hidden)
        self.cond_proj = (nn.Sequential(nn.Linear(cfg.video_cond_dim, cfg.encoder_hidden), nn.SiLU(),
                                        nn.Linear(cfg.encoder_hidden, cfg.encoder_hidden))
                          if cfg.video_cond_dim > 0 else None)
        self.strides = _factorise_ratio(cfg.action_horizon // cfg.num_tokens)
        layers: List[nn.Module] = []
        for s in self.strides:
            layers += [nn.Conv1d(cfg.encoder_hidden, cfg.encoder_hidden, kernel_size=s * 2 - 1,
                                 stride=s, padding=s - 1),
                       nn.GroupNorm(min(8, cfg.encoder_hidden), cfg.encoder_hidden), nn.SiLU(),
                       ResidualConv1dBlock(cfg.encoder_hidden)]
        self.down = nn.Sequential(*layers)
        self.suite_embed = None
        if cfg.num_suites > 0:
            self.suite_embed = nn.Embedding(cfg.num_suites, cfg.encoder_hidden)
            nn.init.zeros_(self.suite_embed.weight)
        self.bottleneck = nn.Linear(cfg.encoder_hidden, cfg.latent_dim * (2 if cfg.variational else 1))


class ActionDecoder(nn.Module):
    """action_ae.py:123-166 (same parameters); forward runs fam_action_decode."""

    def __init__(self, cfg: ActionAEConfig):
        super().__init__()
        self.cfg = cfg
        self.input_proj = nn.Linear(cfg.latent_dim, cfg.decoder_hidden)
        self.strides = _factorise_ratio(cfg.action_horizon // cfg.num_tokens)
        layers: List[nn.Module] = []
        for s in self.strides:
            layers += [nn.ConvTranspose1d(cfg.decoder_hidden, cfg.decoder_hidden, kernel_size=s * 2,
                                          stride=s, padding=s // 2),
                       nn.GroupNorm(min(8, cfg.decoder_hidden), cfg.decoder_hidden), nn.SiLU(),
                       ResidualConv1dBlock(cfg.decoder_hidden)]
        self.up = nn.Sequential(*layers)
        self.output_proj = nn.Linear(cfg.decoder_hidden, cfg.action_dim)
        self.suite_embed = None
        if cfg.num_suites > 0:
            self.suite_embed = nn.Embedding(cfg.num_suites, cfg.decoder_hidden)
            nn.init.zeros_(self.suite_embed.weight)
        # DiT4DiT's decoder (ActionAE.from_dit4dit): latent statistics applied inside the
        # kernels, and task ids required when the decoder holds a task embedding
        self.register_buffer("latent_std", None, persistent=False)
        self.register_buffer("latent_mean", None, persistent=False)
        self.require_suite_ids = False
        self._packed = None
        self.register_load_state_dict_post_hook(lambda m, k: setattr(m, "_packed", None))

    def _apply(self, fn, *args, **kwargs):
        self._packed = None
        return super()._apply(fn, *args, **kwargs)

    def _pack(self):
        dev = self.input_proj.weight.device
        keep: List[torch.Tensor] = []

        def ptr(t):
            t = _f32(t, dev)
            keep.append(t)
            return t.data_ptr()

        stages = (_abi.DecoderStage * len(self.strides))()
        for i, s in enumerate(self.strides):
            ct, gn0, rb = self.up[4 * i], self.up[4 * i + 1], self.up[4 * i + 3].net
            st = stages[i]
            st.convt_w, st.convt_b = ptr(ct.weight), ptr(ct.bias)
            st.gn0_w, st.gn0_b = ptr(gn0.weight), ptr(gn0.bias)
            st.c1_w, st.c1_b = ptr(rb[0].weight), ptr(rb[0].bias)
            st.gn1_w, st.gn1_b = ptr(rb[1].weight), ptr(rb[1].bias)
            st.c2_w, st.c2_b = ptr(rb[3].weight), ptr(rb[3].bias)
            st.gn2_w, st.gn2_b = ptr(rb[4].weight), ptr(rb[4].bias)
            st.stride = s
        w = _abi.DecoderWeights()
        w.in_w, w.in_b = ptr(self.input_proj.weight), ptr(self.input_proj.bias)
        w.out_w, w.out_b = ptr(self.output_proj.weight), ptr(self.output_proj.bias)
        w.suite_embed = ptr(self.suite_embed.weight) if self.suite_embed is not None else None
        w.stages = stages
        w.num_stages = len(self.strides)
        if self.latent_std is not None:
            w.latent_std, w.latent_mean = ptr(self.latent_std), ptr(self.latent_mean)
        c = self.cfg
        cfg = _abi.DecoderConfig(c.action_dim, c.action_horizon, c.num_tokens, c.latent_dim,
                                 c.decoder_hidden, c.num_suites)
        self._packed = (cfg, w, stages, keep)

    def check_ids(self, suite_ids) -> None:
        """DiT4DiT's decoder refuses to run without task ids when it holds a task
        embedding (action_vae.py:168-172); FastWAM's skips the embedding instead."""
        if self.require_suite_ids and suite_ids is None:
            raise ValueError("task_ids are required for a task-conditioned ActionVAE")

    def forward(self, z: torch.Tensor, suite_ids: Optional[torch.Tensor] = None) -> torch.Tensor:
        if not z.is_cuda:
            raise RuntimeError("ActionDecoder runs on CUDA through libfam")
        self.check_ids(suite_ids)
        if self._packed is None:
            self._pack()
        cfg, w, _, _ = self._packed
        zz = z.to(torch.float32).contiguous()
        B = zz.shape[0]
        out = torch.empty((B, self.cfg.action_horizon, self.cfg.action_dim), device=z.device)
        n = C.c_size_t()
        check(lib().fam_decoder_workspace_size(C.byref(cfg), C.byref(w), B, C.byref(n)),
              "fam_decoder_workspace_size")
        ws = torch.empty(n.value, dtype=torch.uint8, device=z.device)
        sid = None
        if suite_ids is not None and self.suite_embed is not None:
            sid = suite_ids.to(device=z.device, dtype=torch.int32).contiguous()
        check(lib().fam_action_decode(C.byref(cfg), C.byref(w), B, zz.data_ptr(),
                                      sid.data_ptr() if sid is not None else None, out.data_ptr(),
                                      ws.data_ptr(), ws.numel(),
                                      C.c_void_p(torch.cuda.current_stream(z.device).cuda_stream)),
              "fam_action_decode")
        return out


class ActionAE(nn.Module):
    """action_ae.py:169-187: same state_dict; decode() on libfam."""

    def __init__(self, cfg: ActionAEConfig):
        super().__init__()
        self.cfg = cfg
        self.encoder = ActionEncoder(cfg)
        self.decoder = ActionDecoder(cfg)

    def decode(self, z: torch.Tensor, suite_ids: Optional[torch.Tensor] = None) -> torch.Tensor:
        return self.decoder(z, suite_ids=suite_ids)

    @classmethod
    def from_dit4dit(cls, checkpoint, map_location="cpu") -> "ActionAE":
        """DiT4DiT's ActionVAE as a decoder (DiT4DiT/model/modules/action_model/action_vae.py:
        136-197), from the checkpoint that load_action_vae reads (action_vae.py:276-283):
        {"config": ActionVAEConfig fields, "model": state_dict}, or a path to one.

        The decoder's task embedding (conditioning_mode "encoder_decoder") loads as the suite
        embedding and task ids become required at decode time, as in DiT4DiT.  When the
        checkpoint sets apply_latent_normalization, its latent_mean / latent_std
        ([num_tokens, latent_dim], std clamped at 1e-4, DiT4DiT/model/framework/DiT4DiT.py:
        256-269) are applied to the latents inside the decode kernels, which is the
        un-normalisation of DiT4DiT._decode_action_predictions (DiT4DiT.py:403-406).
        DiT4DiT runs its encoder only to make training targets, so the returned model has
        encoder None."""
        import os
        if isinstance(checkpoint, (str, os.PathLike)):
            checkpoint = torch.load(checkpoint, map_location=map_location, weights_only=False)
        c = dict(checkpoint["config"])
        num_tasks = int(c.get("num_tasks", 0))
        mode = c.get("conditioning_mode") or ("encoder_decoder" if num_tasks > 0 else "none")
        if mode not in ("none", "encoder_only", "encoder_decoder"):
            raise ValueError(f"conditioning_mode must be one of none, encoder_only, encoder_decoder; got {mode!r}")
        if mode != "none" and num_tasks <= 0:
            raise ValueError(f"conditioning_mode={mode!r} requires num_tasks > 0")
        horizon, tokens = int(c.get("action_horizon", 16)), int(c.get("num_tokens", 4))
        if horizon % tokens:
            raise ValueError(f"action_horizon must be divisible by num_tokens, got {horizon} and {tokens}")
        cfg = ActionAEConfig(action_dim=int(c.get("action_dim", 29)), action_horizon=horizon, num_tokens=tokens,
                             latent_dim=int(c.get("latent_dim", 64)), encoder_hidden=int(c.get("encoder_hidden", 128)),
                             decoder_hidden=int(c.get("decoder_hidden", 128)), video_cond_dim=0,
                             variational=bool(c.get("variational", True)),
                             num_suites=num_tasks if mode == "encoder_decoder" else 0)
        ae = cls.__new__(cls)
        nn.Module.__init__(ae)
        ae.cfg = cfg
        ae.encoder = None
        ae.decoder = ActionDecoder(cfg)
        sd = {}
        for k, v in checkpoint["model"].items():
            if k.startswith("decoder."):
                k = k[len("decoder."):]
                sd["suite_embed.weight" if k == "task_embedding.weight" else k] = v.float()
        ae.decoder.load_state_dict(sd, strict=True)
        ae.decoder.require_suite_ids = cfg.num_suites > 0
        if checkpoint.get("apply_latent_normalization", False):
            shape = (cfg.num_tokens, cfg.latent_dim)
            mean = checkpoint.get("latent_mean", torch.zeros(shape)).float()
            std = checkpoint.get("latent_std", torch.ones(shape)).float().clamp_min(1e-4)
            while mean.dim() > 2 and mean.shape[0] == 1:
                mean = mean[0]
            while std.dim() > 2 and std.shape[0] == 1:
                std = std[0]
            ae.decoder.latent_mean = torch.broadcast_to(mean, shape).contiguous()
            ae.decoder.latent_std = torch.broadcast_to(std, shape).contiguous()
        return ae


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
