"""The bounded mbarrier wait of the tensor-core kernels gives up and reports, and the context survives.

Every pipeline wait in fastmd_b200/csrc/gemm_tcgen05.cu is bounded (about a second); on expiry the CTA
raises FMD_FLAG_WAIT_TIMEOUT instead of hanging. ``fmd_wait_probe`` runs that same wait on a barrier
nothing arrives at (no copy or MMA in flight), so the expiry is exercised without faulting or hanging the
GPU; a wide GEMM afterwards must still run and be right."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

FLAG_WAIT_TIMEOUT = 64


def test_bounded_wait_expires_and_reports(cuda):
    from fastmd_b200 import wide_gemm
    from fastmd_b200._lib import call, ptr, stream

    flags = torch.zeros(1, dtype=torch.int32, device=cuda)
    call("fmd_wait_probe", 1, ptr(flags), stream(cuda))  # the barrier completes: no flag
    torch.cuda.synchronize()
    assert int(flags.item()) == 0
    t0 = time.perf_counter()
    call("fmd_wait_probe", 0, ptr(flags), stream(cuda))  # nothing arrives: the wait must give up
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert int(flags.item()) == FLAG_WAIT_TIMEOUT
    assert 0.5 < elapsed < 30.0
    # the context is usable: a tcgen05 GEMM after the expired wait
    gen = torch.Generator(device=cuda).manual_seed(0)
    x = torch.randn((1000, 256), device=cuda, generator=gen)
    w = torch.randn((128, 256), device=cuda, generator=gen) / 16
    y = wide_gemm.linear(x, w)
    ref = (x.double() @ w.double().T)
    assert float((y.double() - ref).abs().max()) < 1e-4
