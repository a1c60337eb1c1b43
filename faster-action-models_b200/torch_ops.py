"""torch.library custom operators over the libfam entry points.

The reference reaches this path through ``torch.library.custom_op("fastwam::<name>",
mutates_args=...)`` plus ``register_fake``, called inside ``torch.compile(mode=
"reduce-overhead", fullgraph=True)`` regions (src/cae-fastwam/.../mot.py:2793-2829;
FastWAM/src/fastwam/models/wan22/fastwam.py:1208-1225).  These operators give the same
boundary over this library:

  fam::prefill_video_cache              MoT.prefill_video_cache_tensor (mot.py:474-526)
  fam::denoise_action_with_video_cache  FastWAM._denoise_action_with_video_cache
                                        (fastwam.py:771-804)
  fam::action_chunk                     the Euler loop of FastWAM.infer_action
                                        (fastwam.py:1241-1263)
  fam::action_decode                    ActionAE.decode (action_ae.py:184-187)

A module holding packed weights is registered once (`register`) and named by an
integer handle, so the operators take tensors and scalars only.  Timesteps are host
scalars (float / List[float], already the values the reference computes in its
dtype): the kernels take them as launch arguments, so no operator reads a device
tensor back to the host, and a call never synchronises the stream.  Every output is
a new tensor (no aliasing of inputs); the fake implementations give shapes, dtypes
and devices from the registered module's configuration, so the operators trace under
FakeTensorMode / torch.compile(fullgraph=True) without running a kernel.
"""
import itertools
from typing import Dict, List, Optional

import torch

from .models import ActionAE, ActionDiT, WanVideoDiT

_modules: Dict[int, object] = {}
_handles = itertools.count(1)


def register(module) -> int:
    """Register a WanVideoDiT, ActionDiT or ActionAE; returns its operator handle."""
    if not isinstance(module, (WanVideoDiT, ActionDiT, ActionAE)):
        raise TypeError(f"cannot register {type(module).__name__}")
    h = next(_handles)
    _modules[h] = module
    return h


def unregister(handle: int) -> None:
    _modules.pop(handle, None)


def _get(handle: int, kind):
    m = _modules.get(handle)
    if m is None or not isinstance(m, kind):
        raise ValueError(f"no {kind.__name__} registered under handle {handle}")
    return m


def _or_none(ts: List[torch.Tensor]) -> Optional[List[torch.Tensor]]:
    return list(ts) if len(ts) > 0 else None


# ------------------------------------------------------------ video prefill
@torch.library.custom_op("fam::prefill_video_cache", mutates_args=())
def prefill_video_cache(handle: int, latents: torch.Tensor, timestep: List[float], context: torch.Tensor,
                        context_mask: Optional[torch.Tensor]) -> List[torch.Tensor]:
    """Per-block K then per-block V ([B, S, H*d] bf16 each, 2 x num_layers tensors);
    timestep: one value per sample, or one for the batch."""
    vid = _get(handle, WanVideoDiT)
    k, v = vid.engine().prefill(latents, list(timestep), context, context_mask)
    return list(k) + list(v)


@prefill_video_cache.register_fake
def _(handle, latents, timestep, context, context_mask):
    vid = _get(handle, WanVideoDiT)
    B, _, Fr, Hh, Ww = latents.shape
    pt, ph, pw = vid.patch_size
    S = (Fr // pt) * (Hh // ph) * (Ww // pw)
    HD = vid.num_heads * vid.attn_head_dim
    return [latents.new_empty((B, S, HD), dtype=torch.bfloat16) for _ in range(2 * vid.num_layers)]


# ------------------------------------------------------------ action expert
@torch.library.custom_op("fam::denoise_action_with_video_cache", mutates_args=())
def denoise_action_with_video_cache(handle: int, latents: torch.Tensor, timestep: float,
                                    context: torch.Tensor, context_mask: Optional[torch.Tensor],
                                    cache_k: List[torch.Tensor], cache_v: List[torch.Tensor],
                                    attn_mask: Optional[torch.Tensor]) -> torch.Tensor:
    """One model evaluation: the velocity [B, Sa, A] (bf16).  Empty cache lists: no video K/V."""
    act = _get(handle, ActionDiT)
    return act.engine().denoise_step(latents, float(timestep), context, context_mask, _or_none(cache_k),
                                     _or_none(cache_v), attn_mask)


@denoise_action_with_video_cache.register_fake
def _(handle, latents, timestep, context, context_mask, cache_k, cache_v, attn_mask):
    _get(handle, ActionDiT)
    return latents.new_empty(latents.shape, dtype=torch.bfloat16)


@torch.library.custom_op("fam::action_chunk", mutates_args=())
def action_chunk(handle: int, latents: torch.Tensor, timesteps: List[float], deltas: List[float],
                 context: torch.Tensor, context_mask: Optional[torch.Tensor], cache_k: List[torch.Tensor],
                 cache_v: List[torch.Tensor], attn_mask: Optional[torch.Tensor]) -> torch.Tensor:
    """len(timesteps) Euler steps from `latents`; the final latents [B, Sa, A] (bf16)."""
    if len(timesteps) != len(deltas) or len(timesteps) == 0:
        raise ValueError("action_chunk: timesteps and deltas must be non-empty and of equal length")
    act = _get(handle, ActionDiT)
    return act.engine().chunk(latents, timesteps, deltas, context, context_mask, _or_none(cache_k),
                              _or_none(cache_v), attn_mask)


@action_chunk.register_fake
def _(handle, latents, timesteps, deltas, context, context_mask, cache_k, cache_v, attn_mask):
    _get(handle, ActionDiT)
    return latents.new_empty(latents.shape, dtype=torch.bfloat16)


# ------------------------------------------------------------ action VAE decode
@torch.library.custom_op("fam::action_decode", mutates_args=())
def action_decode(handle: int, z: torch.Tensor, suite_ids: Optional[torch.Tensor]) -> torch.Tensor:
    """Action latents [B, num_tokens, latent_dim] -> chunk [B, action_horizon, action_dim] (fp32)."""
    return _get(handle, ActionAE).decode(z, suite_ids)


@action_decode.register_fake
def _(handle, z, suite_ids):
    cfg = _get(handle, ActionAE).cfg
    return z.new_empty((z.shape[0], cfg.action_horizon, cfg.action_dim), dtype=torch.float32)
