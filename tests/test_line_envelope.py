"""The MatRIS line-graph envelope product: the oracle against the reference's kernels (golden, CPU) and
``fmd_matris_line_envelope(_bwd)`` against both (GPU): forward bitwise, backward to 2e-6 relative (the
reference adds its rows with float atomics in launch order, this build in each bond's CSR order)."""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import line_envelope as ole


@pytest.mark.parametrize("tag", ["small", "wide"])
def test_oracle_equals_reference_kernels(tag):
    g = golden("line_envelope")
    base, src, tgt, gout = (g[f"env_{tag}_{k}"] for k in ("base", "source", "target", "gout"))
    assert np.array_equal(ole.forward(base, src, tgt), g[f"env_{tag}_out"])
    assert np.array_equal(ole.backward(gout, base, src, tgt), g[f"env_{tag}_grad"])


@pytest.mark.gpu
@pytest.mark.parametrize("tag", ["small", "wide"])
def test_line_envelope_kernels_equal_the_reference(cuda, tag):
    from fastmd_b200._lib import call, flags_word, ptr, stream
    from fastmd_b200.ops import segment_csr

    g = golden("line_envelope")
    base, src, tgt, gout = (g[f"env_{tag}_{k}"] for k in ("base", "source", "target", "gout"))
    U, D = base.shape
    T = src.shape[0]
    lg = np.zeros((T, 5), np.int32)
    lg[:, 1], lg[:, 3] = tgt, src  # column 1 the target bond, column 3 the source bond
    tb, tl = torch.from_numpy(base).to(cuda), torch.from_numpy(lg).to(cuda)
    env = torch.empty((T, D), device=cuda)
    call("fmd_matris_line_envelope", ptr(tb), D, ptr(tl), T, U, D, ptr(env), D, ptr(flags_word(cuda)), stream(cuda))
    p1, o1 = segment_csr(torch.from_numpy(tgt).to(cuda), U)
    p2, o2 = segment_csr(torch.from_numpy(src).to(cuda), U)
    tg = torch.from_numpy(gout).to(cuda)
    grad = torch.empty((U, D), device=cuda)
    call("fmd_matris_line_envelope_bwd", ptr(tb), D, ptr(tl), U, D, ptr(tg), D, ptr(p1), ptr(o1), ptr(p2), ptr(o2),
         ptr(grad), D, stream(cuda))
    torch.cuda.synchronize()
    assert np.array_equal(env.cpu().numpy(), g[f"env_{tag}_out"])
    ref = g[f"env_{tag}_grad"]
    assert np.abs(grad.cpu().numpy() - ref).max() <= 2e-6 * np.abs(ref).max()
