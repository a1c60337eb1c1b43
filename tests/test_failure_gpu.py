"""Failure path on the GPU without a fault: a bounded device wait that nothing
completes gives up after its 1 s %globaltimer limit, records its code in the
device status word and returns; the context stays usable (a GEMM through the
ABI afterwards still matches torch)."""
import ctypes as C
import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu

L = importlib.import_module("faster-action-models_b200._lib")
ops = importlib.import_module("faster-action-models_b200.ops")


def test_bounded_wait_reports_and_context_survives():
    st = torch.cuda.current_stream().cuda_stream
    L.device_status(st, reset=True)  # start clean
    L.check(L.lib().fam_selftest_bounded_wait(C.c_void_p(st)), "fam_selftest_bounded_wait")
    torch.cuda.synchronize()
    assert L.device_status(st, reset=True) == 1  # a consumer wait expired
    assert L.device_status(st, reset=False) == 0  # reset took effect
    g = torch.Generator().manual_seed(0)
    x = torch.randn(32, 256, generator=g).bfloat16().cuda()
    w = torch.randn(384, 256, generator=g).bfloat16().cuda()
    y = ops.gemm(w, x, weights_as_a=True)
    torch.cuda.synchronize()
    ref = (x.float() @ w.float().t())
    assert (y.float() - ref).abs().max().item() <= 2e-2 * max(1.0, ref.abs().max().item())
    assert L.device_status(st, reset=False) == 0
