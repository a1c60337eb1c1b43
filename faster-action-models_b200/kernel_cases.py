"""Fixed single-GPU workloads of the library's kernels, for profilers.

    python faster-action-models_b200/kernel_cases.py {gemm_qkv_c2,attn_c2,cae_c0} [repeats]

Each case runs its library call `repeats` times (default 3) on cuda:0 and
synchronizes; under ncu, skip the warm-up launches with `-s`.
  gemm_qkv_c2  ops.gemm: [1760, 3072] x [9216, 3072]^T + bias (backbone qkv, config 2)
  attn_c2      ops.attention: 1760 tokens, 24 heads x 128, first-frame-causal (352)
  cae_c0       CAEEngine.chunk + ActionAE.decode of BASELINE config 0
"""
import importlib
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
ops = importlib.import_module("faster-action-models_b200.ops")
M = importlib.import_module("faster-action-models_b200.models")


def main(case: str, reps: int) -> None:
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    if case == "gemm_qkv_c2":
        a = torch.randn(1760, 3072, device=dev).bfloat16()
        w = (torch.randn(9216, 3072, device=dev) * 0.02).bfloat16()
        b = torch.randn(9216, device=dev).bfloat16()
        for _ in range(reps):
            ops.gemm(a, w, bias=b)
    elif case == "attn_c2":
        q, k, v = (torch.randn(1, 1760, 24 * 128, device=dev).bfloat16() for _ in range(3))
        for _ in range(reps):
            ops.attention(q, k, v, 24, first_frame_tokens=352)
    elif case == "cae_c0":
        dit = M.ActionDiT(hidden_dim=32, action_dim=16, ffn_dim=128, text_dim=3072, freq_dim=256, eps=1e-6,
                          num_heads=4, attn_head_dim=8, num_layers=8).to(dev)
        ae = M.ActionAE(M.ActionAEConfig(action_dim=7, action_horizon=32, num_tokens=8, latent_dim=16,
                                         decoder_hidden=256, video_cond_dim=0, variational=True)).to(dev)
        ctx = torch.randn(1, 512, 3072, device=dev)
        noise = torch.randn(1, 8, 16, device=dev)
        ts, ds = M.build_inference_schedule(4, 1.0, dtype=torch.float32)
        eng = dit.engine()
        for _ in range(reps):
            ae.decode(eng.chunk(noise, ts, ds, ctx))
    else:
        raise SystemExit(f"unknown case {case!r}")
    torch.cuda.synchronize()
    print("ok", case)


if __name__ == "__main__":
    main(sys.argv[1], int(sys.argv[2]) if len(sys.argv) > 2 else 3)
