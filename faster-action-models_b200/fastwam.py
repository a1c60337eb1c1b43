"""The FastWAM policy object and its MoT core on the libfam path.

Mirrors the reference's model-level interface for the per-action-chunk path:

  FastWAM.infer_action          FastWAM/src/fastwam/models/wan22/fastwam.py:1080-1274
  FastWAM._denoise_action_with_video_cache                  fastwam.py:771-804
  FastWAM._encode_input_image_latents_tensor                fastwam.py:296-306
  FastWAM._append_proprio_to_context                        fastwam.py:257-278
  FastWAM._build_mot_attention_mask                         fastwam.py:429-451
  FastWAM.decode_action_latents                             fastwam.py:855-863
  FastWAM.save_checkpoint / load_checkpoint                 fastwam.py:1300-1345
  MoT (mixtures "video" / "action")                         mot.py:18-60
  MoT.prefill_video_cache_tensor                            mot.py:474-526
  MoT.forward_action_with_video_cache_tensor                mot.py:528-578
  infer_action_multi            eval/native/fastwam_batched_infer.py:23-122

Same argument names, defaults, validation errors and return values; the checkpoint
payload is the reference's ({"mot": mot.state_dict(), "proprio_encoder": ...} with
`mixtures.video.` / `mixtures.action.` keys), so reference checkpoints load unchanged.

Every stage runs in libfam: the observation's VAE encode (vae.py), the video prefill
into the per-layer K/V cache, the action expert's Euler loop (one fused persistent
kernel per chunk at batch 1) and the Action-VAE decode.  The reference's prepare
stages (patch / action embedding, time MLPs, text embedding) are fused into those
kernels, so WanVideoDiT.prepare / ActionDiT.prepare return records that carry the
stage inputs (models.PreparedVideo / PreparedAction) in the reference's tuple slots,
and the MoT methods run the fused kernels from them.  The call graph is the
reference's: infer_action calls `self.mot.prefill_video_cache_tensor` and, when
`_denoise_action_with_video_cache` (or `mot.forward_action_with_video_cache_tensor`)
is replaced on the instance -- as the reference's perf and oracle harnesses do
(geak/task/scripts/episode_perf.py:248-312) -- every Euler step goes through the
replacement; otherwise the whole loop is one fused chunk.
"""
from __future__ import annotations

from typing import Any, Optional, Sequence, Union

import torch
import torch.nn.functional as F
from torch import nn

from .models import (ActionAE, ActionDiT, ActionStepOut, PreparedAction, PreparedVideo, WanVideoDiT,
                     build_inference_schedule)
from .pipeline import visible_video_prefix


class WanContinuousFlowMatchScheduler:
    """Host-side flow-matching schedule (schedulers/scheduler_continuous.py:22-88)."""

    def __init__(self, num_train_timesteps: int = 1000, shift: float = 5.0):
        self.num_train_timesteps = int(num_train_timesteps)
        self.shift = float(shift)

    def build_inference_schedule(self, num_inference_steps: int, device=None, dtype=torch.float32,
                                 shift_override: Optional[float] = None):
        """(timesteps [N], deltas [N]) as host tensors in `dtype` (the kernels take the
        values as launch arguments, so the schedule never lives on the device)."""
        shift = self.shift if shift_override is None else float(shift_override)
        ts, ds = build_inference_schedule(num_inference_steps, shift, dtype=dtype,
                                          num_train_timesteps=self.num_train_timesteps)
        return torch.tensor(ts, dtype=dtype), torch.tensor(ds, dtype=dtype)

    def step(self, model_output, delta, sample):
        """x + v * delta in the sample's dtype (scheduler_continuous.py:82-88)."""
        d = delta.to(dtype=sample.dtype, device=sample.device) if torch.is_tensor(delta) else delta
        return sample + model_output * d


class MoT(nn.Module):
    """Mixture-of-Transformers holder (mot.py:18-60): `mixtures` with a "video" and an
    "action" expert of equal depth, heads and head width; state_dict keys
    `mixtures.video.*` / `mixtures.action.*`."""

    def __init__(self, mixtures: dict, mot_checkpoint_mixed_attn: bool = False):
        super().__init__()
        if not mixtures:
            raise ValueError("`mixtures` cannot be empty.")
        if "video" not in mixtures or "action" not in mixtures:
            raise ValueError("`mixtures` must include both 'video' and 'action' experts.")
        if mot_checkpoint_mixed_attn:
            raise ValueError("mixed-attention gradient checkpointing is a training feature, not on this path")
        self.mixtures = nn.ModuleDict(mixtures)
        self.expert_order = list(self.mixtures.keys())
        first = self.mixtures[self.expert_order[0]]
        self.num_layers = len(first.blocks)
        self.num_heads = first.num_heads
        self.attn_head_dim = first.attn_head_dim
        for name in self.expert_order[1:]:
            e = self.mixtures[name]
            if len(e.blocks) != self.num_layers:
                raise ValueError(f"All experts must have same number of layers; got {self.num_layers} and "
                                 f"{len(e.blocks)}")
            if e.num_heads != self.num_heads:
                raise ValueError(f"All experts must have same num_heads; got {self.num_heads} and {e.num_heads}")
            if e.attn_head_dim != self.attn_head_dim:
                raise ValueError("All experts must have same attn_head_dim; "
                                 f"got {self.attn_head_dim} and {e.attn_head_dim}")

    def prefill_video_cache_tensor(self, video_tokens, video_freqs, video_t_mod, video_context,
                                   video_context_mask, video_attention_mask):
        """MoT.prefill_video_cache_tensor (mot.py:474-526): the video expert's blocks over the
        prepared video, caching each block's K (after RMSNorm + RoPE) and V.  video_tokens is
        the record WanVideoDiT.prepare returned; the self-attention mask is the expert's
        video_attention_mask_mode (first-frame causal on the policy path), which the kernels
        apply themselves.  Returns (list of K, list of V), [B, S, H*d] bf16 each."""
        if not isinstance(video_tokens, PreparedVideo):
            raise TypeError("prefill_video_cache_tensor takes the record returned by WanVideoDiT.prepare "
                            "(the token stage runs fused inside the prefill kernels)")
        vid = self.mixtures["video"]
        return vid.engine().prefill(video_tokens.latents, video_tokens.timestep, video_tokens.context,
                                    video_tokens.context_mask)

    def forward_action_with_video_cache_tensor(self, action_tokens, action_freqs, action_t_mod, action_context,
                                               action_context_mask, video_cache_k, video_cache_v,
                                               action_attention_mask):
        """MoT.forward_action_with_video_cache_tensor (mot.py:528-578): the action expert's
        blocks, each with joint attention of the action queries over [cached video K/V ;
        action K/V] under action_attention_mask ([Sa, Sv + Sa]).  action_tokens is the
        record ActionDiT.prepare returned; the step kernels end with the head, so the
        result is an ActionStepOut that ActionDiT.post unwraps."""
        if not isinstance(action_tokens, PreparedAction):
            raise TypeError("forward_action_with_video_cache_tensor takes the record returned by "
                            "ActionDiT.prepare (the token stage runs fused inside the step kernels)")
        act = self.mixtures["action"]
        vel = act.engine().denoise_step(action_tokens.latents, action_tokens.timestep, action_tokens.context,
                                        action_tokens.context_mask, video_cache_k, video_cache_v,
                                        action_attention_mask)
        return ActionStepOut(vel)


class FastWAM(nn.Module):
    """MoT world model with video / action experts (fastwam.py:21-118), inference side."""

    def __init__(self, video_expert: WanVideoDiT, action_expert: ActionDiT, mot: MoT, vae, text_encoder=None,
                 tokenizer=None, text_dim: Optional[int] = None, proprio_dim: Optional[int] = None,
                 action_vae: Optional[ActionAE] = None, action_vae_suite_id: Optional[int] = None,
                 device: str = "cuda", torch_dtype: torch.dtype = torch.bfloat16, video_train_shift: float = 5.0,
                 video_infer_shift: float = 5.0, video_num_train_timesteps: int = 1000,
                 action_train_shift: float = 5.0, action_infer_shift: float = 5.0,
                 action_num_train_timesteps: int = 1000, loss_lambda_video: float = 1.0,
                 loss_lambda_action: float = 1.0, compile_training_denoise: bool = False):
        super().__init__()
        self.video_expert = video_expert
        self.action_expert = action_expert
        self.mot = mot
        self.dit = self.mot
        self.vae = vae
        self.action_vae = action_vae
        self.action_vae_suite_id = action_vae_suite_id
        if self.action_vae is not None:
            self.action_vae.eval()
            self.action_vae.requires_grad_(False)
        self.text_encoder = text_encoder
        self.tokenizer = tokenizer
        if text_dim is None:
            if self.text_encoder is None:
                raise ValueError("`text_dim` is required when `text_encoder` is not loaded.")
            text_dim = int(self.text_encoder.dim)
        self.text_dim = int(text_dim)
        self.proprio_dim = None if proprio_dim is None else int(proprio_dim)
        self.proprio_encoder = (nn.Linear(self.proprio_dim, self.text_dim).to(torch_dtype)
                                if self.proprio_dim is not None else None)
        self.train_video_scheduler = WanContinuousFlowMatchScheduler(video_num_train_timesteps, video_train_shift)
        self.infer_video_scheduler = WanContinuousFlowMatchScheduler(video_num_train_timesteps, video_infer_shift)
        self.train_action_scheduler = WanContinuousFlowMatchScheduler(action_num_train_timesteps, action_train_shift)
        self.infer_action_scheduler = WanContinuousFlowMatchScheduler(action_num_train_timesteps, action_infer_shift)
        self.train_scheduler = self.train_video_scheduler
        self.infer_scheduler = self.infer_video_scheduler
        self.device = torch.device(device)
        self.torch_dtype = torch_dtype
        self.loss_lambda_video = float(loss_lambda_video)
        self.loss_lambda_action = float(loss_lambda_action)
        self.compile_training_denoise = bool(compile_training_denoise)
        self.to(self.device)

    def to(self, *args, **kwargs):
        super().to(*args, **kwargs)
        if self.vae is not None and hasattr(self.vae, "to"):
            self.vae.to(*args, **kwargs)
        return self

    # ------------------------------------------------------------ stages
    @torch.no_grad()
    def encode_prompt(self, prompt: Union[str, Sequence[str]]):
        """fastwam.py:240-255: tokenizer + text encoder, padding zeroed, an all-ones mask."""
        if self.text_encoder is None or self.tokenizer is None:
            raise ValueError("Prompt encoding requires loaded text encoder/tokenizer. "
                             "Set `load_text_encoder=true` or provide precomputed `context/context_mask`.")
        ids, mask = self.tokenizer(prompt, return_mask=True, add_special_tokens=True)
        ids, mask = ids.to(self.device), mask.to(self.device, dtype=torch.bool)
        emb = self.text_encoder(ids, mask)
        seq_lens = mask.gt(0).sum(dim=1).long()
        for i, v in enumerate(seq_lens):
            emb[i, v:] = 0
        return emb.to(device=self.device), torch.ones_like(mask)

    def _append_proprio_to_context(self, context, context_mask, proprio):
        if self.proprio_encoder is None or proprio is None:
            return context, context_mask
        if proprio.ndim != 2:
            raise ValueError(f"`proprio` must be 2D [B, D], got shape {tuple(proprio.shape)}")
        if self.proprio_dim is None or proprio.shape[1] != self.proprio_dim:
            raise ValueError(f"`proprio` last dim must be {self.proprio_dim}, got {proprio.shape[1]}")
        w, b = self.proprio_encoder.weight, self.proprio_encoder.bias
        token = F.linear(proprio.to(device=self.device, dtype=context.dtype).unsqueeze(1), w.to(context.dtype),
                         None if b is None else b.to(context.dtype)).to(dtype=context.dtype)
        ones = torch.ones((context_mask.shape[0], 1), dtype=torch.bool, device=context_mask.device)
        return torch.cat([context, token], dim=1), torch.cat([context_mask, ones], dim=1)

    @torch.no_grad()
    def _encode_input_image_latents_tensor(self, input_image: torch.Tensor, tiled=False, tile_size=(30, 52),
                                           tile_stride=(15, 26)):
        if input_image.ndim == 3:
            input_image = input_image.unsqueeze(0)
        if input_image.ndim != 4 or input_image.shape[0] != 1 or input_image.shape[1] != 3:
            raise ValueError(f"`input_image` must have shape [1,3,H,W] or [3,H,W], got {tuple(input_image.shape)}")
        if tiled:
            raise NotImplementedError("Batched VAE image encoding does not support tiled encoding.")
        image = input_image.to(device=self.device)[0].unsqueeze(1)
        return self.vae.model.encode(image.unsqueeze(0), self.vae.scale)

    @torch.no_grad()
    def _build_mot_attention_mask(self, video_seq_len: int, action_seq_len: int, video_tokens_per_frame: int,
                                  device) -> torch.Tensor:
        total = video_seq_len + action_seq_len
        mask = torch.zeros((total, total), dtype=torch.bool, device=device)
        mask[:video_seq_len, :video_seq_len] = self.video_expert.build_video_to_video_mask(
            video_seq_len=video_seq_len, video_tokens_per_frame=video_tokens_per_frame, device=device)
        mask[video_seq_len:, video_seq_len:] = True
        mask[video_seq_len:, :min(video_tokens_per_frame, video_seq_len)] = True
        return mask

    def _denoise_action_with_video_cache(self, latents_action, timestep_action, context, context_mask,
                                         video_cache_k, video_cache_v, action_attention_mask):
        """One model evaluation of the action expert over the video cache -> velocity
        [B, Sa, A] (bf16).  A timestep tensor on the GPU is read back once per call; the
        policy loop hands host values."""
        tokens, _t, t_mod, a_ctx, a_cm, freqs = self.action_expert.prepare(
            action_tokens=latents_action, timestep=timestep_action, context=context, context_mask=context_mask)
        tokens = self.mot.forward_action_with_video_cache_tensor(
            action_tokens=tokens, action_freqs=freqs, action_t_mod=t_mod, action_context=a_ctx,
            action_context_mask=a_cm, video_cache_k=video_cache_k, video_cache_v=video_cache_v,
            action_attention_mask=action_attention_mask)
        return self.action_expert.post(tokens)

    def _action_vae_suite_ids(self, batch: int, device):
        if self.action_vae_suite_id is None:
            return None
        return torch.full((batch,), int(self.action_vae_suite_id), dtype=torch.long, device=device)

    def decode_action_latents(self, latents: torch.Tensor) -> torch.Tensor:
        """Action latent tokens -> chunk (fp32 Action-VAE, cast back to the model dtype);
        a model without an Action-VAE returns the latents."""
        if self.action_vae is None:
            return latents
        suite_ids = self._action_vae_suite_ids(latents.shape[0], latents.device)
        return self.action_vae.decode(latents.to(dtype=torch.float32), suite_ids=suite_ids).to(dtype=self.torch_dtype)

    def _step_replaced(self) -> bool:
        return ("_denoise_action_with_video_cache" in self.__dict__
                or "forward_action_with_video_cache_tensor" in self.mot.__dict__
                or "prepare" in self.action_expert.__dict__ or "post" in self.action_expert.__dict__)

    # ------------------------------------------------------------ entry point
    @torch.no_grad()
    def infer_action(self, prompt: Optional[str], input_image: torch.Tensor, action_horizon: int,
                     proprio: Optional[torch.Tensor] = None, context: Optional[torch.Tensor] = None,
                     context_mask: Optional[torch.Tensor] = None, negative_prompt: Optional[str] = None,
                     text_cfg_scale: float = 1.0, num_inference_steps: int = 20, sigma_shift: Optional[float] = None,
                     seed: Optional[int] = None, rand_device: str = "cpu", tiled: bool = False,
                     compile_action_infer: bool = False, return_action_latents: bool = False) -> dict[str, Any]:
        """FastWAM.infer_action (fastwam.py:1080-1274).  compile_action_infer is accepted:
        the library captures its prefill and chunk launches in CUDA graphs itself.
        Returns {"action": [T, A] fp32 CPU} (+ "action_latents")."""
        self.eval()
        if str(getattr(self.video_expert, "video_attention_mask_mode", "")) != "first_frame_causal":
            raise ValueError("`infer_action` requires `video_attention_mask_mode='first_frame_causal'`.")
        if input_image.ndim == 3:
            input_image = input_image.unsqueeze(0)
        if input_image.ndim != 4 or input_image.shape[0] != 1 or input_image.shape[1] != 3:
            raise ValueError(f"`input_image` must have shape [1,3,H,W] or [3,H,W], got {tuple(input_image.shape)}")
        _, _, height, width = input_image.shape
        if height % 16 != 0 or width % 16 != 0:
            raise ValueError("`input_image` must be resized before infer, expected multiples of 16 but got "
                             f"HxW=({height},{width})")
        if proprio is not None:
            if self.proprio_dim is None:
                raise ValueError("`proprio` was provided but `proprio_dim=None` so `proprio_encoder` is disabled.")
            if proprio.ndim == 1:
                proprio = proprio.unsqueeze(0)
            elif not (proprio.ndim == 2 and proprio.shape[0] == 1):
                raise ValueError(f"`proprio` must be [D] or [1,D], got shape {tuple(proprio.shape)}")
            if proprio.shape[1] != self.proprio_dim:
                raise ValueError(f"`proprio` last dim must be {self.proprio_dim}, got {proprio.shape[1]}")
            proprio = proprio.to(device=self.device, dtype=self.torch_dtype)
        generator = None if seed is None else torch.Generator(device=rand_device).manual_seed(seed)
        latent_horizon = self.action_vae.cfg.num_tokens if self.action_vae is not None else action_horizon
        latents_action = torch.randn((1, latent_horizon, self.action_expert.action_dim), generator=generator,
                                     device=rand_device, dtype=torch.float32).to(device=self.device,
                                                                                 dtype=self.torch_dtype)
        input_image = input_image.to(device=self.device, dtype=self.torch_dtype)
        first_frame_latents = self._encode_input_image_latents_tensor(input_image=input_image, tiled=tiled)
        fuse_flag = bool(getattr(self.video_expert, "fuse_vae_embedding_in_latents", False))
        use_prompt = prompt is not None
        use_context = context is not None or context_mask is not None
        if use_prompt and use_context:
            raise ValueError("`prompt` and `context/context_mask` are mutually exclusive.")
        if not use_prompt and not use_context:
            raise ValueError("Either `prompt` or both `context/context_mask` must be provided.")
        if use_prompt:
            context, context_mask = self.encode_prompt(prompt)
        else:
            if context is None or context_mask is None:
                raise ValueError("`context` and `context_mask` must be both provided together.")
            if context.ndim == 2:
                context = context.unsqueeze(0)
            if context_mask.ndim == 1:
                context_mask = context_mask.unsqueeze(0)
            if context.ndim != 3 or context_mask.ndim != 2:
                raise ValueError(f"`context/context_mask` must be [B,L,D]/[B,L], got {tuple(context.shape)} and "
                                 f"{tuple(context_mask.shape)}")
            context = context.to(device=self.device, dtype=self.torch_dtype, non_blocking=True)
            context_mask = context_mask.to(device=self.device, dtype=torch.bool, non_blocking=True)
        if proprio is not None:
            context, context_mask = self._append_proprio_to_context(context=context, context_mask=context_mask,
                                                                    proprio=proprio)
        timestep_video = torch.zeros((first_frame_latents.shape[0],), dtype=torch.float32)
        (video_tokens, _t_video, video_t_mod, video_context, video_context_mask, video_freqs, _f, _h, _w,
         tokens_per_frame) = self.video_expert.prepare(
            x=first_frame_latents, timestep=timestep_video, context=context, context_mask=context_mask,
            action=None, fuse_vae_embedding_in_latents=fuse_flag)
        video_seq_len = int(video_tokens.shape[1])
        attention_mask = self._build_mot_attention_mask(video_seq_len=video_seq_len,
                                                        action_seq_len=latents_action.shape[1],
                                                        video_tokens_per_frame=tokens_per_frame, device=self.device)
        video_cache_k, video_cache_v = self.mot.prefill_video_cache_tensor(
            video_tokens=video_tokens, video_freqs=video_freqs, video_t_mod=video_t_mod, video_context=video_context,
            video_context_mask=video_context_mask, video_attention_mask=attention_mask[:video_seq_len, :video_seq_len])
        action_attention_mask = attention_mask[video_seq_len:, :]
        ts, ds = self.infer_action_scheduler.build_inference_schedule(
            num_inference_steps=num_inference_steps, device=self.device, dtype=latents_action.dtype,
            shift_override=sigma_shift)
        if self._step_replaced():
            # a harness replaced a stage on the instance: every Euler step goes through it
            for step_t, step_delta in zip(ts, ds):
                pred = self._denoise_action_with_video_cache(
                    latents_action=latents_action, timestep_action=step_t.unsqueeze(0), context=context,
                    context_mask=context_mask, video_cache_k=video_cache_k, video_cache_v=video_cache_v,
                    action_attention_mask=action_attention_mask)
                latents_action = self.infer_action_scheduler.step(pred, step_delta, latents_action)
        else:
            # the whole loop as one fused chunk over the cache rows the MoT mask leaves visible
            kv, vv, sv = visible_video_prefix(video_cache_k, video_cache_v, tokens_per_frame)
            vis_mask = torch.cat([action_attention_mask[:, :sv], action_attention_mask[:, video_seq_len:]], dim=1)
            latents_action = self.action_expert.engine().chunk(
                latents_action, ts.float().tolist(), ds.float().tolist(), context, context_mask, kv, vv, vis_mask)
        output = {"action": self.decode_action_latents(latents_action)[0].detach().to(device="cpu",
                                                                                       dtype=torch.float32)}
        if return_action_latents:
            output["action_latents"] = latents_action[0].detach().to(device="cpu", dtype=torch.float32)
        return output

    # ------------------------------------------------------------ checkpoints
    def save_checkpoint(self, path, optimizer=None, step=None):
        payload = {"mot": self.mot.state_dict(), "step": step, "torch_dtype": str(self.torch_dtype)}
        if self.proprio_encoder is not None:
            payload["proprio_encoder"] = self.proprio_encoder.state_dict()
        if optimizer is not None:
            payload["optimizer"] = optimizer.state_dict()
        torch.save(payload, path)

    def load_checkpoint(self, path, optimizer=None):
        """The reference payload ({"mot": ..., "proprio_encoder": ...}, or a legacy
        {"dit": ...} for the video expert alone) from a path or an already-loaded dict."""
        payload = path if isinstance(path, dict) else torch.load(path, map_location="cpu")
        if "mot" in payload:
            self.mot.load_state_dict(payload["mot"], strict=False)
        elif "dit" in payload:
            self.video_expert.load_state_dict(payload["dit"], strict=False)
        else:
            raise ValueError(f"Checkpoint missing both `mot` and `dit` keys: {path if not isinstance(path, dict) else '<dict>'}")
        if self.proprio_encoder is not None and "proprio_encoder" in payload:
            self.proprio_encoder.load_state_dict(payload["proprio_encoder"], strict=True)
        for expert in (self.video_expert, self.action_expert):
            expert._engine = None  # repack the new weights on the next call
        if optimizer is not None and "optimizer" in payload:
            optimizer.load_state_dict(payload["optimizer"])
        return payload


@torch.no_grad()
def infer_action_multi(model: FastWAM, prompts, input_images, action_horizon: int, proprios,
                       num_inference_steps: int, sigma_shift: Optional[float] = None,
                       seeds: Optional[Sequence[int]] = None, rand_device: str = "cpu", tiled: bool = False,
                       context: Optional[torch.Tensor] = None, context_mask: Optional[torch.Tensor] = None):
    """Batched twin of FastWAM.infer_action for B distinct observations
    (eval/native/fastwam_batched_infer.py:23-122): per-row noise from one generator per
    seed over `action_horizon` rows, VAE encode of every observation, prompts encoded
    (once when identical), proprio tokens, the prefill and the Euler loop at batch B.
    Returns {"action": the final action latents [B, action_horizon, A]} like the reference.
    A host without a text encoder passes `context` / `context_mask` ([B, L, D] / [B, L])
    instead of prompts."""
    model.eval()
    if str(getattr(model.video_expert, "video_attention_mask_mode", "")) != "first_frame_causal":
        raise ValueError("requires video_attention_mask_mode='first_frame_causal'")
    if input_images.ndim != 4 or input_images.shape[1] != 3:
        raise ValueError(f"input_images must be [B,3,H,W], got {tuple(input_images.shape)}")
    B, _, height, width = input_images.shape
    if height % 16 or width % 16:
        raise ValueError(f"H,W must be multiples of 16, got {height}x{width}")
    if context is None and len(prompts) != B:
        raise ValueError(f"{len(prompts)} prompts for B={B}")
    device, dtype = model.device, model.torch_dtype
    if seeds is None:
        seeds = [None] * B
    rows = []
    for s in seeds:
        g = None if s is None else torch.Generator(device=rand_device).manual_seed(int(s))
        rows.append(torch.randn((1, action_horizon, model.action_expert.action_dim), generator=g,
                                device=rand_device, dtype=torch.float32))
    latents_action = torch.cat(rows, dim=0).to(device=device, dtype=dtype)
    x = input_images.to(device=device, dtype=dtype)
    first_frame_latents = torch.cat([model.vae.model.encode(x[i].unsqueeze(1).unsqueeze(0), model.vae.scale)
                                     for i in range(B)], dim=0)
    if context is None:
        if len(set(prompts)) == 1:
            c1, m1 = model.encode_prompt(prompts[0])
            context = c1.repeat(B, *([1] * (c1.ndim - 1)))
            context_mask = m1.repeat(B, *([1] * (m1.ndim - 1)))
        else:
            cs, ms = zip(*(model.encode_prompt(p) for p in prompts))
            context, context_mask = torch.cat(list(cs), 0), torch.cat(list(ms), 0)
    else:
        context = context.to(device=device, dtype=dtype)
        context_mask = context_mask.to(device=device, dtype=torch.bool)
    if proprios is not None:
        context, context_mask = model._append_proprio_to_context(
            context=context, context_mask=context_mask, proprio=proprios.to(device=device, dtype=dtype))
    (video_tokens, _t, video_t_mod, video_context, video_context_mask, video_freqs, _f, _h, _w,
     tokens_per_frame) = model.video_expert.prepare(x=first_frame_latents, timestep=torch.zeros(B),
                                                     context=context, context_mask=context_mask)
    video_seq_len = int(video_tokens.shape[1])
    mask = model._build_mot_attention_mask(video_seq_len, latents_action.shape[1], tokens_per_frame, device)
    cache_k, cache_v = model.mot.prefill_video_cache_tensor(
        video_tokens=video_tokens, video_freqs=video_freqs, video_t_mod=video_t_mod, video_context=video_context,
        video_context_mask=video_context_mask, video_attention_mask=mask[:video_seq_len, :video_seq_len])
    ts, ds = model.infer_action_scheduler.build_inference_schedule(
        num_inference_steps=num_inference_steps, device=device, dtype=latents_action.dtype, shift_override=sigma_shift)
    kv, vv, sv = visible_video_prefix(cache_k, cache_v, tokens_per_frame)
    amask = mask[video_seq_len:, :]
    vis_mask = torch.cat([amask[:, :sv], amask[:, video_seq_len:]], dim=1)
    latents_action = model.action_expert.engine().chunk(latents_action, ts.float().tolist(), ds.float().tolist(),
                                                        context, context_mask, kv, vv, vis_mask)
    return {"action": latents_action}
