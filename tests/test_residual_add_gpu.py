"""The residual add (fmd_residual_add) against the reference kernels' golden outputs and the oracle.

Bar: bitwise (one rounded product and one rounded addition per element, the reference's order)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import residual_add as ora

pytestmark = pytest.mark.gpu
GOLDEN = np.load(Path(__file__).parent / "golden" / "residual_add.npz")


@pytest.mark.parametrize("tag", ["d128", "d64_strided", "d5"])
def test_golden_bitwise_with_autograd(tag):
    from fastmd_b200.residual_add import residual_add

    n, d, sd, sr = (int(v) for v in GOLDEN[f"ra_{tag}_meta"])
    # the leaves are the wide buffers; row-strided column views of them are read in place
    delta_base = torch.from_numpy(GOLDEN[f"ra_{tag}_delta"]).cuda().requires_grad_(True)
    residual_base = torch.from_numpy(GOLDEN[f"ra_{tag}_residual"]).cuda().requires_grad_(True)
    weight = torch.from_numpy(GOLDEN[f"ra_{tag}_weight"]).cuda().reshape(1, d)
    out = residual_add(delta_base[:, :d], residual_base[:, :d], weight)
    assert out.is_contiguous() and out.shape == (n, d)
    np.testing.assert_array_equal(out.detach().cpu().numpy(), GOLDEN[f"ra_{tag}_out"])
    out.backward(torch.from_numpy(GOLDEN[f"ra_{tag}_gout"]).cuda())
    np.testing.assert_array_equal(delta_base.grad[:, :d].cpu().numpy(), GOLDEN[f"ra_{tag}_gout"])
    np.testing.assert_array_equal(residual_base.grad[:, :d].cpu().numpy(), GOLDEN[f"ra_{tag}_gres"])
    assert torch.all(delta_base.grad[:, d:] == 0) and torch.all(residual_base.grad[:, d:] == 0)


@pytest.mark.parametrize("n,d", [(155_648, 128), (3001, 7), (1, 1), (0, 16)])
def test_matches_oracle(n, d):
    from fastmd_b200.residual_add import residual_add

    g = torch.Generator().manual_seed(n + d)
    delta, residual, weight = torch.randn(n, d, generator=g), torch.randn(n, d, generator=g), torch.randn(d, generator=g)
    out = residual_add(delta.cuda(), residual.cuda(), weight.cuda())
    np.testing.assert_array_equal(out.cpu().numpy(), ora.forward(delta.numpy(), residual.numpy(), weight.numpy()))


def test_non_unit_column_stride_is_copied_and_misaligned_rows_take_the_scalar_path():
    from fastmd_b200.residual_add import residual_add

    g = torch.Generator(device="cuda").manual_seed(3)
    wide = torch.randn(64, 40, device="cuda", generator=g)
    delta = wide.t()[:, :64]  # [40, 64] with column stride 40
    residual = torch.randn(41 * 64 + 1, device="cuda", generator=g)[1:].reshape(41, 64)[:40]  # 4-byte offset
    weight = torch.randn(64, device="cuda", generator=g)
    out = residual_add(delta, residual, weight)
    ref = ora.forward(delta.cpu().numpy(), residual.cpu().numpy(), weight.cpu().numpy())
    np.testing.assert_array_equal(out.cpu().numpy(), ref)
