"""Policy-level entry points built from the libfam engines.

FastWAMActionPolicy.infer_action follows FastWAM.infer_action
(FastWAM/src/fastwam/models/wan22/fastwam.py:1080-1274) from the first-frame
latents on: seeded CPU noise, video prefill at timestep 0 into the per-block
K/V cache, the MoT attention mask (action rows see the first video frame and
every action token, fastwam.py:429-451), the flow-matching Euler loop of the
action expert over the cache, and the optional Action-VAE decode, returning
the chunk as fp32 on the CPU.  The observation VAE encode that produces the
first-frame latents, and prompt encoding, are outside this path.

FastWAMJointPolicy.infer_joint follows FastWAM.infer_joint (fastwam.py:866-1078):
video and action latents denoised together.  Under the MoT mask the video rows
attend only to video keys, so each model evaluation (_joint_denoise_core,
fastwam.py:492-554) is the video expert's own forward over the current noisy
video latents -- whose per-block K/V is that step's cache -- plus its output
head, and the action expert over that cache.

FastWAMJointPolicy(action_sees_full_video=True) is FastWAMJoint
(fastwam_joint.py:29-49): the action rows attend to the whole video.
FastWAMIDMPolicy.infer_action follows FastWAMIDM.infer_action
(fastwam_idm.py:365-589): the video is denoised alone first (_denoise_video,
:283-313: the video expert and its head, first frame pinned), then prefilled at
timestep 0 into the K/V cache, and the action Euler loop runs over that cache
with the FastWAMJoint mask.

CAEPipeline is BASELINE config 4: the video backbone forward once per chunk,
the compact action expert cross-attending the backbone's final token states,
and the Action-VAE decoder, over a batch of independent rollouts processed in
micro-batches.

DiT4DiTPipeline is BASELINE config 3 (the DiT4DiT world action model restated
with the FastWAM classes): the backbone runs only up to its feature block (tail
elision, `elide_backbone`) and a flow-matching action head cross-attends that
block's token states.
"""
from __future__ import annotations

import copy
from typing import Optional, Sequence

import torch
from torch import nn

from .models import ActionAE, ActionDiT, WanVideoDiT, build_inference_schedule


def visible_video_prefix(cache_k, cache_v, tokens_per_frame: int):
    """The cache rows the action tokens can see under the MoT mask: the first video
    frame only (fastwam.py:429-451).  The keys after it are masked for every action row,
    so the action expert attends over this prefix (strided views, no copy) with an
    all-attend mask and gets the same result without streaming the masked keys."""
    vis = min(tokens_per_frame, cache_k[0].shape[1])
    return [t[:, :vis] for t in cache_k], [t[:, :vis] for t in cache_v], vis


def mot_action_mask(video_seq_len: int, action_seq_len: int, tokens_per_frame: int,
                    device=None) -> torch.Tensor:
    """Action rows [Sa, Sv + Sa] of FastWAM._build_mot_attention_mask (fastwam.py:429-451):
    every action token, and the first video frame only."""
    m = torch.zeros(action_seq_len, video_seq_len + action_seq_len, dtype=torch.uint8, device=device)
    m[:, video_seq_len:] = 1
    m[:, :min(tokens_per_frame, video_seq_len)] = 1
    return m


class FastWAMActionPolicy:
    def __init__(self, video_expert: WanVideoDiT, action_expert: ActionDiT,
                 action_vae: Optional[ActionAE] = None, action_infer_shift: float = 5.0,
                 torch_dtype=torch.bfloat16):
        if video_expert.num_heads != action_expert.num_heads or \
                video_expert.attn_head_dim != action_expert.attn_head_dim or \
                video_expert.num_layers != action_expert.num_layers:
            raise ValueError("experts must share layer count, heads and head dim (mot.py:38-52)")
        self.video_expert = video_expert
        self.action_expert = action_expert
        self.action_vae = action_vae
        self.shift = float(action_infer_shift)
        self.torch_dtype = torch_dtype
        self.device = next(action_expert.parameters()).device

    @torch.no_grad()
    def _denoise_action_with_video_cache(self, latents_action: torch.Tensor, timestep_action,
                                         context: torch.Tensor, context_mask, video_cache_k, video_cache_v,
                                         action_attention_mask) -> torch.Tensor:
        """FastWAM._denoise_action_with_video_cache (fastwam.py:771-804): one model evaluation of
        the action expert over the video K/V cache; the velocity [B, Sa, A].  An instance may
        replace this attribute; infer_action then runs its Euler loop through the replacement."""
        return self.action_expert.engine().denoise_step(latents_action, timestep_action, context, context_mask,
                                                        video_cache_k, video_cache_v, action_attention_mask)

    @torch.no_grad()
    def infer_action(self, first_frame_latents: torch.Tensor, context: torch.Tensor,
                     context_mask: torch.Tensor, action_horizon: int, num_inference_steps: int = 20,
                     sigma_shift: Optional[float] = None, seed: Optional[int] = None,
                     return_action_latents: bool = False) -> dict:
        vid, act = self.video_expert, self.action_expert
        gen = None if seed is None else torch.Generator(device="cpu").manual_seed(seed)
        latent_horizon = self.action_vae.cfg.num_tokens if self.action_vae is not None else action_horizon
        noise = torch.randn((1, latent_horizon, act.action_dim), generator=gen, dtype=torch.float32)
        lat = noise.to(device=self.device, dtype=self.torch_dtype)
        # video prefill at timestep 0 (fastwam.py:1175-1234)
        k, v = vid.prefill(first_frame_latents, torch.zeros(first_frame_latents.shape[0]), context,
                           context_mask)
        pt, ph, pw = vid.patch_size
        tpf = (first_frame_latents.shape[3] // ph) * (first_frame_latents.shape[4] // pw)
        k, v, Sv = visible_video_prefix(k, v, tpf)
        mask = mot_action_mask(Sv, latent_horizon, tpf, device=self.device)
        ts, ds = build_inference_schedule(num_inference_steps,
                                          self.shift if sigma_shift is None else float(sigma_shift),
                                          dtype=self.torch_dtype)
        if "_denoise_action_with_video_cache" in self.__dict__:
            # the step was replaced on this instance (as the reference's perf / oracle
            # harnesses do): run the Euler loop through it, one model evaluation per step
            for t, d in zip(ts, ds):
                tt = torch.full((lat.shape[0],), float(t), dtype=self.torch_dtype)
                vel = self._denoise_action_with_video_cache(lat, tt, context, context_mask, k, v, mask)
                lat = (lat + vel * float(d)).to(self.torch_dtype)
        else:
            lat = act.engine().chunk(lat, ts, ds, context, context_mask, k, v, mask)
        out = {}
        if self.action_vae is not None:
            out["action"] = self.action_vae.decode(lat.float())[0].to(dtype=self.torch_dtype).float().cpu()
        else:
            out["action"] = lat[0].float().cpu()
        if return_action_latents:
            out["action_latents"] = lat[0].float().cpu()
        return out


class FastWAMJointPolicy(FastWAMActionPolicy):
    """FastWAM.infer_joint from the first-frame latents on (video decode excluded).
    action_sees_full_video: the FastWAMJoint mask (action rows attend to every video
    token) instead of FastWAM's (the first frame only)."""

    def __init__(self, video_expert: WanVideoDiT, action_expert: ActionDiT,
                 action_vae: Optional[ActionAE] = None, action_infer_shift: float = 5.0,
                 video_infer_shift: float = 5.0, torch_dtype=torch.bfloat16,
                 action_sees_full_video: bool = False):
        super().__init__(video_expert, action_expert, action_vae, action_infer_shift, torch_dtype)
        self.video_shift = float(video_infer_shift)
        self.full_video = bool(action_sees_full_video)

    def _action_view(self, k, v, Sa: int, tpf: int):
        """The cache rows and action mask of the action half of a step."""
        if self.full_video:
            Sv = k[0].shape[1]
            return k, v, torch.ones(Sa, Sv + Sa, dtype=torch.uint8, device=self.device)
        kv, vv, Sv = visible_video_prefix(k, v, tpf)
        return kv, vv, mot_action_mask(Sv, Sa, tpf, device=self.device)

    @torch.no_grad()
    def video_step(self, latents_video: torch.Tensor, timestep_video, context: torch.Tensor,
                   context_mask: torch.Tensor, return_cache: bool = False):
        """The video expert alone over the current latents plus its output head
        (FastWAMIDM._denoise_video) -> bf16 [B, C, F, H, W] (and the step's K/V)."""
        vid = self.video_expert
        eng = vid.engine()
        B, _, Fr, Hh, Ww = latents_video.shape
        pt, ph, pw = vid.patch_size
        grid = (Fr // pt, Hh // ph, Ww // pw)
        t_rows = torch.empty(B, 2, vid.hidden_dim, dtype=torch.bfloat16, device=self.device)
        k, v, hidden = eng.prefill(latents_video, timestep_video, context, context_mask, return_hidden=True,
                                   use_graph=False, t_out=t_rows)
        pred = eng.post(hidden, t_rows, grid, grid[1] * grid[2])
        return (pred, k, v) if return_cache else pred

    @torch.no_grad()
    def joint_step(self, latents_video: torch.Tensor, latents_action: torch.Tensor, timestep_video,
                   timestep_action, context: torch.Tensor, context_mask: torch.Tensor):
        """FastWAM._joint_denoise_core -> (video prediction bf16 [B, C, F, H, W],
        action prediction bf16 [B, Sa, A])."""
        vid, act = self.video_expert, self.action_expert
        pt, ph, pw = vid.patch_size
        tpf = (latents_video.shape[3] // ph) * (latents_video.shape[4] // pw)
        pred_video, k, v = self.video_step(latents_video, timestep_video, context, context_mask, return_cache=True)
        kv, vv, mask = self._action_view(k, v, latents_action.shape[1], tpf)
        pred_action = act.engine().denoise_step(latents_action, timestep_action, context, context_mask, kv, vv, mask)
        return pred_video, pred_action

    @torch.no_grad()
    def infer_joint(self, first_frame_latents: torch.Tensor, num_latent_frames: int, context: torch.Tensor,
                    context_mask: torch.Tensor, action_horizon: int, num_inference_steps: int = 20,
                    sigma_shift: Optional[float] = None, seed: Optional[int] = None) -> dict:
        """Seeded CPU noise for both latents (fastwam.py:945-965), the first latent frame
        pinned to the observation after every step (:1063), both Euler updates in bf16
        (scheduler_continuous.py:82-88).  Returns {"video_latents", "action"}."""
        act = self.action_expert
        B, zc, _, lh, lw = first_frame_latents.shape
        gv = None if seed is None else torch.Generator(device="cpu").manual_seed(seed)
        ga = None if seed is None else torch.Generator(device="cpu").manual_seed(seed)
        lat_v = torch.randn((1, zc, num_latent_frames, lh, lw), generator=gv, dtype=torch.float32).to(
            device=self.device, dtype=self.torch_dtype)
        latent_horizon = self.action_vae.cfg.num_tokens if self.action_vae is not None else action_horizon
        lat_a = torch.randn((1, latent_horizon, act.action_dim), generator=ga, dtype=torch.float32).to(
            device=self.device, dtype=self.torch_dtype)
        first = first_frame_latents.to(device=self.device, dtype=self.torch_dtype)
        lat_v[:, :, 0:1] = first
        ts_v, ds_v = build_inference_schedule(num_inference_steps, self.video_shift if sigma_shift is None
                                              else float(sigma_shift), dtype=self.torch_dtype)
        ts_a, ds_a = build_inference_schedule(num_inference_steps, self.shift if sigma_shift is None
                                              else float(sigma_shift), dtype=self.torch_dtype)
        for tv, dv, ta, da in zip(ts_v, ds_v, ts_a, ds_a):
            pv, pa = self.joint_step(lat_v, lat_a, torch.tensor([tv]), torch.tensor([ta]), context, context_mask)
            lat_v = lat_v + pv * torch.tensor(dv, dtype=self.torch_dtype, device=self.device)
            lat_a = lat_a + pa * torch.tensor(da, dtype=self.torch_dtype, device=self.device)
            lat_v[:, :, 0:1] = first
        out = {"video_latents": lat_v}
        if self.action_vae is not None:
            out["action"] = self.action_vae.decode(lat_a.float())[0].to(dtype=self.torch_dtype).float().cpu()
        else:
            out["action"] = lat_a[0].float().cpu()
        return out


class FastWAMIDMPolicy(FastWAMJointPolicy):
    """FastWAMIDM.infer_action from the first-frame latents on: the video denoised
    alone, then the actions over its timestep-0 cache (the action rows see the whole
    video, FastWAMJoint's mask)."""

    def __init__(self, video_expert: WanVideoDiT, action_expert: ActionDiT,
                 action_vae: Optional[ActionAE] = None, action_infer_shift: float = 5.0,
                 video_infer_shift: float = 5.0, torch_dtype=torch.bfloat16):
        super().__init__(video_expert, action_expert, action_vae, action_infer_shift, video_infer_shift,
                         torch_dtype, action_sees_full_video=True)

    @torch.no_grad()
    def infer_action(self, first_frame_latents: torch.Tensor, num_latent_frames: int, context: torch.Tensor,
                     context_mask: torch.Tensor, action_horizon: int, num_inference_steps: int = 20,
                     sigma_shift: Optional[float] = None, seed: Optional[int] = None) -> dict:
        """Returns {"video_latents", "action"} (fastwam_idm.py:365-589; the reference's
        action latents are the action horizon itself: no Action-VAE in this model)."""
        vid, act = self.video_expert, self.action_expert
        B, zc, _, lh, lw = first_frame_latents.shape
        gv = None if seed is None else torch.Generator(device="cpu").manual_seed(seed)
        ga = None if seed is None else torch.Generator(device="cpu").manual_seed(seed)
        lat_v = torch.randn((1, zc, num_latent_frames, lh, lw), generator=gv, dtype=torch.float32).to(
            device=self.device, dtype=self.torch_dtype)
        lat_a = torch.randn((1, action_horizon, act.action_dim), generator=ga, dtype=torch.float32).to(
            device=self.device, dtype=self.torch_dtype)
        first = first_frame_latents.to(device=self.device, dtype=self.torch_dtype)
        lat_v[:, :, 0:1] = first
        ts_v, ds_v = build_inference_schedule(num_inference_steps, self.video_shift if sigma_shift is None
                                              else float(sigma_shift), dtype=self.torch_dtype)
        for tv, dv in zip(ts_v, ds_v):
            pv = self.video_step(lat_v, torch.tensor([tv]), context, context_mask)
            lat_v = lat_v + pv * torch.tensor(dv, dtype=self.torch_dtype, device=self.device)
            lat_v[:, :, 0:1] = first
        k, v = vid.prefill(lat_v, torch.zeros(lat_v.shape[0]), context, context_mask)
        Sv = k[0].shape[1]
        mask = torch.ones(action_horizon, Sv + action_horizon, dtype=torch.uint8, device=self.device)
        ts_a, ds_a = build_inference_schedule(num_inference_steps, self.shift if sigma_shift is None
                                              else float(sigma_shift), dtype=self.torch_dtype)
        lat_a = act.engine().chunk(lat_a, ts_a, ds_a, context, context_mask, k, v, mask)
        return {"video_latents": lat_v, "action": lat_a[0].float().cpu()}


class FastWAMOptionalIDMPolicy(FastWAMIDMPolicy):
    """FastWAMOptionalIDM.infer_action (fastwam_optional_idm.py:60-120): "idm" runs the
    IDM path, "first_frame" FastWAM's (the actions over the first frame's cache)."""

    @torch.no_grad()
    def infer_action(self, first_frame_latents: torch.Tensor, context: torch.Tensor, context_mask: torch.Tensor,
                     action_horizon: int, num_inference_steps: int = 20, sigma_shift: Optional[float] = None,
                     seed: Optional[int] = None, num_latent_frames: Optional[int] = None,
                     action_infer_mode: str = "idm") -> dict:
        if action_infer_mode == "idm":
            if num_latent_frames is None:
                raise ValueError("num_latent_frames is required for action_infer_mode='idm'")
            return FastWAMIDMPolicy.infer_action(self, first_frame_latents, num_latent_frames, context, context_mask,
                                                 action_horizon, num_inference_steps, sigma_shift, seed)
        if action_infer_mode == "first_frame":
            return FastWAMActionPolicy.infer_action(self, first_frame_latents, context, context_mask, action_horizon,
                                                    num_inference_steps, sigma_shift, seed)
        raise ValueError("action_infer_mode must be one of: idm, first_frame")


class CAEPipeline:
    """backbone forward -> compact expert over its final token states ->
    Action-VAE decode, for a batch of rollouts in micro-batches."""

    def __init__(self, video: WanVideoDiT, expert: ActionDiT, ae: ActionAE, num_steps: int = 4,
                 shift: float = 1.0, micro_batch: int = 16):
        if not expert.is_compact():
            raise ValueError("CAEPipeline expects a compact (hidden <= 64) action expert")
        if expert.text_dim != video.hidden_dim:
            raise ValueError("the expert's text_dim must equal the backbone hidden width")
        self.video, self.expert, self.ae = video, expert, ae
        self.ts, self.ds = build_inference_schedule(num_steps, shift, dtype=torch.float32)
        self.micro_batch = micro_batch
        self._bufs = {}

    def _buffers(self, b: int, S: int, dev):
        """Per micro-batch size: the K/V cache the prefill writes (the attention source of
        every block) and the final token states, allocated once so that the captured
        launch graphs replay."""
        key = (b, S)
        if key not in self._bufs:
            v = self.video
            HD = v.num_heads * v.attn_head_dim
            ks = [torch.empty(b, S, HD, dtype=torch.bfloat16, device=dev) for _ in range(v.num_layers)]
            vs = [torch.empty(b, S, HD, dtype=torch.bfloat16, device=dev) for _ in range(v.num_layers)]
            hid = torch.empty(b, S, v.hidden_dim, dtype=torch.float32, device=dev)
            self._bufs[key] = (ks, vs, hid)
        return self._bufs[key]

    @torch.no_grad()
    def __call__(self, latents: torch.Tensor, timestep, context: torch.Tensor,
                 context_mask: Optional[torch.Tensor], noise: torch.Tensor) -> torch.Tensor:
        """latents [B, in, F, H, W], noise [B, num_tokens, latent_dim] -> actions [B, horizon, A]."""
        B = latents.shape[0]
        outs = []
        t = timestep if torch.is_tensor(timestep) else torch.full((B,), float(timestep))
        t = t.reshape(-1)
        if t.numel() == 1:
            t = t.expand(B)
        for s in range(0, B, self.micro_batch):
            e = min(B, s + self.micro_batch)
            cm = context_mask[s:e] if context_mask is not None else None
            pt, ph, pw = self.video.patch_size
            S = (latents.shape[2] // pt) * (latents.shape[3] // ph) * (latents.shape[4] // pw)
            ks, vs, hid = self._buffers(e - s, S, latents.device)
            _, _, hidden = self.video.engine().prefill(latents[s:e], t[s:e], context[s:e], cm,
                                                       return_hidden=True, cache_k=ks, cache_v=vs,
                                                       hidden=hid)
            # Euler loop + Action-VAE decode (the decode in the step kernel's epilogue)
            _, actions = self.expert.engine().chunk_decode(noise[s:e].to(hidden.device, torch.float32),
                                                           self.ts, self.ds, hidden, self.ae)
            outs.append(actions)
        return torch.cat(outs)


def elide_backbone(video: WanVideoDiT, extract_layer: int) -> WanVideoDiT:
    """A WanVideoDiT that shares `video`'s parameters but holds blocks 0..extract_layer
    only: its prefill returns the token states after block `extract_layer` (the
    feature hook of DiT4DiT, Cosmos25.py:152-171 with extract_layer 17 in
    DiT4DiT/config/libero/dit4dit_libero.yaml:14), and the later blocks never run."""
    if not 0 <= extract_layer < video.num_layers:
        raise ValueError(f"extract_layer {extract_layer} outside 0..{video.num_layers - 1}")
    el = copy.copy(video)
    el._modules = dict(video._modules)
    el._modules["blocks"] = nn.ModuleList(list(video.blocks)[:extract_layer + 1])
    el._engine = None
    return el


class DiT4DiTPipeline:
    """backbone features at `extract_layer` -> flow-matching action head
    (ActionDiT cross-attending the features, no video cache) over `num_steps` Euler steps
    -> optional Action-VAE decode, in micro-batches.

    A compact head (hidden <= 64) runs the fp32 compact engine and denoises action
    latents for the decoder; a wide head runs the bf16 action-expert engine and
    returns the denoised chunk itself (decoded when `ae` is given)."""

    def __init__(self, video: WanVideoDiT, head: ActionDiT, extract_layer: int,
                 ae: Optional[ActionAE] = None, num_steps: int = 4, shift: float = 1.0,
                 micro_batch: int = 16):
        if head.text_dim != video.hidden_dim:
            raise ValueError("the head's text_dim must equal the backbone hidden width")
        self.backbone = elide_backbone(video, extract_layer)
        self.head, self.ae = head, ae
        self.ts, self.ds = build_inference_schedule(num_steps, shift, dtype=torch.float32)
        self.micro_batch = micro_batch
        self._bufs = {}

    def _buffers(self, b: int, S: int, dev):
        key = (b, S)
        if key not in self._bufs:
            v = self.backbone
            HD = v.num_heads * v.attn_head_dim
            ks = [torch.empty(b, S, HD, dtype=torch.bfloat16, device=dev) for _ in range(v.num_layers)]
            vs = [torch.empty(b, S, HD, dtype=torch.bfloat16, device=dev) for _ in range(v.num_layers)]
            hid = torch.empty(b, S, v.hidden_dim, dtype=torch.float32, device=dev)
            self._bufs[key] = (ks, vs, hid)
        return self._bufs[key]

    @torch.no_grad()
    def __call__(self, latents: torch.Tensor, timestep, context: torch.Tensor,
                 context_mask: Optional[torch.Tensor], noise: torch.Tensor) -> torch.Tensor:
        """latents [B, in, F, H, W], noise [B, Sa, A] -> fp32 [B, Sa, A] (or decoded actions)."""
        B = latents.shape[0]
        t = timestep if torch.is_tensor(timestep) else torch.full((B,), float(timestep))
        t = t.reshape(-1)
        if t.numel() == 1:
            t = t.expand(B)
        pt, ph, pw = self.backbone.patch_size
        S = (latents.shape[2] // pt) * (latents.shape[3] // ph) * (latents.shape[4] // pw)
        outs = []
        for s in range(0, B, self.micro_batch):
            e = min(B, s + self.micro_batch)
            cm = context_mask[s:e] if context_mask is not None else None
            ks, vs, hid = self._buffers(e - s, S, latents.device)
            _, _, feats = self.backbone.engine().prefill(latents[s:e], t[s:e], context[s:e], cm,
                                                         return_hidden=True, cache_k=ks, cache_v=vs,
                                                         hidden=hid)
            if self.head.is_compact() and self.ae is not None:
                _, actions = self.head.engine().chunk_decode(noise[s:e].to(feats.device, torch.float32),
                                                             self.ts, self.ds, feats, self.ae)
                outs.append(actions)
                continue
            if self.head.is_compact():
                lat = self.head.engine().chunk(noise[s:e].to(feats.device, torch.float32),
                                               self.ts, self.ds, feats)
            else:
                lat = self.head.engine().chunk(noise[s:e].to(feats.device, torch.bfloat16),
                                               self.ts, self.ds, feats).float()
            outs.append(self.ae.decode(lat) if self.ae is not None else lat)
        return torch.cat(outs)
