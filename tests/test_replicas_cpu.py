"""Multi-process (gloo, world size 2) checks of the batch-sharding host logic: shards
cover the batch exactly once, per-rollout seeding does not depend on the sharding, and
the gathered shard results equal the single-process result (the decode runs through the
CPU oracle here; on GPUs each rank runs the libfam path on its own device)."""
import importlib
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

R = importlib.import_module("faster-action-models_b200.replicas")


def test_shard_range_partitions():
    for total in (0, 1, 7, 16, 1024, 1025):
        for world in (1, 2, 3, 4, 8):
            spans = [R.shard_range(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        R.shard_range(4, 2, 2)


def test_seeded_noise_is_per_rollout():
    full = R.seeded_noise(range(10), (8, 16))
    part = R.seeded_noise(range(4, 7), (8, 16))
    assert torch.equal(full[4:7], part)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, total, out_q):
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import torch.distributed as dist
    from datetime import timedelta
    from oracle import fam_oracle as O
    Rm = importlib.import_module("faster-action-models_b200.replicas")
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    torch.manual_seed(0)
    Mm = importlib.import_module("faster-action-models_b200.models")
    ae = Mm.ActionAE(Mm.ActionAEConfig(action_dim=7, action_horizon=32, num_tokens=8, latent_dim=16,
                                       decoder_hidden=32, video_cond_dim=0))
    sd = {k: v.float() for k, v in ae.state_dict().items()}
    cfg = O.DecoderConfig(7, 32, 8, 16, 32)

    def fn(start, stop):
        z = Rm.seeded_noise(range(start, stop), (8, 16))
        return O.action_decode(sd, cfg, z)

    parts = Rm.run_shard(fn, total, world, rank)
    t = Rm.max_over_ranks(float(rank + 1))
    if rank == 0:
        out_q.put((torch.cat([p for p in parts if p.numel()]), t))
    dist.barrier()
    dist.destroy_process_group()


def test_gloo_two_ranks_match_single_process():
    total, world = 7, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, total, q)) for r in range(world)]
    for p in procs:
        p.start()
    got, tmax = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    from oracle import fam_oracle as O
    M = importlib.import_module("faster-action-models_b200.models")
    torch.manual_seed(0)
    ae = M.ActionAE(M.ActionAEConfig(action_dim=7, action_horizon=32, num_tokens=8, latent_dim=16,
                                     decoder_hidden=32, video_cond_dim=0))
    sd = {k: v.float() for k, v in ae.state_dict().items()}
    ref = O.action_decode(sd, O.DecoderConfig(7, 32, 8, 16, 32), R.seeded_noise(range(total), (8, 16)))
    # CPU convolutions may reassociate with the batch size: fp32-rounding tolerance
    assert got.shape == ref.shape and torch.allclose(got, ref, atol=1e-5, rtol=1e-5)
    assert tmax == 2.0
