"""fmd_pair_aggregate through the reference surface against the reference's kernels (golden vectors,
bitwise) and the oracle at a larger size; strided inputs, autograd, the index-range flag."""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import pair_aggregate as opa

pytestmark = pytest.mark.gpu
CASES = ["d32", "d128_strided", "d5"]


@pytest.mark.parametrize("tag", CASES)
def test_pair_aggregate_golden_bitwise(tag):
    from fastmd_b200.pair_aggregate import directed_pair_average, undirected_pair_expand

    z = golden("pair_aggregate")
    g = {k[len(f"pa_{tag}_"):]: z[k] for k in z if k.startswith(f"pa_{tag}_")}
    U, D, stride = (int(v) for v in g["meta"])
    pair = torch.from_numpy(g["pair"]).cuda()
    # the data are the first D columns of a [2U, stride] buffer, read in place
    base = torch.from_numpy(g["base"]).cuda().requires_grad_(True)
    avg = directed_pair_average(base[:, :D], pair)
    np.testing.assert_array_equal(avg.detach().cpu().numpy(), g["avg"])
    avg.backward(torch.from_numpy(g["gavg"]).cuda())
    np.testing.assert_array_equal(base.grad.cpu().numpy()[:, :D], g["gdata"])

    und = torch.from_numpy(g["und"]).cuda().requires_grad_(True)
    exp = undirected_pair_expand(und[:, :D], pair, 2 * U)
    np.testing.assert_array_equal(exp.detach().cpu().numpy(), g["exp"])
    exp.backward(torch.from_numpy(g["gexp"]).cuda())
    np.testing.assert_array_equal(und.grad.cpu().numpy()[:, :D], g["gund"])


@pytest.mark.parametrize("U,D,idx", [(60889, 128, torch.int64), (5001, 64, torch.int32), (777, 3, torch.int64),
                                     (1, 1, torch.int64)])
def test_pair_aggregate_oracle(U, D, idx):
    from fastmd_b200.pair_aggregate import directed_pair_average, undirected_pair_expand

    rng = np.random.default_rng(U + D)
    seg = np.repeat(np.arange(U), 2)[rng.permutation(2 * U)]
    pair = np.argsort(seg, kind="stable").reshape(U, 2)
    x = rng.standard_normal((2 * U, D)).astype(np.float32)
    y = rng.standard_normal((U, D)).astype(np.float32)
    pd = torch.from_numpy(pair).to(idx).cuda()
    np.testing.assert_array_equal(directed_pair_average(torch.from_numpy(x).cuda(), pd).cpu().numpy(),
                                  opa.average(x, pair))
    np.testing.assert_array_equal(undirected_pair_expand(torch.from_numpy(y).cuda(), pd, 2 * U).cpu().numpy(),
                                  opa.expand(y, pair, 2 * U))


def test_empty_and_index_flag():
    from fastmd_b200 import _lib
    from fastmd_b200._lib import call, ptr, stream
    from fastmd_b200.pair_aggregate import directed_pair_average, undirected_pair_expand

    empty = torch.empty((0, 2), dtype=torch.int64, device="cuda")
    assert directed_pair_average(torch.empty((0, 8), device="cuda"), empty).shape == (0, 8)
    assert undirected_pair_expand(torch.empty((0, 8), device="cuda"), empty, 0).shape == (0, 8)
    # a pair naming row 9 of 4 directed rows: flagged, the gathered row reads as zero
    flags = torch.zeros(1, dtype=torch.int32, device="cuda")
    bad = torch.tensor([[0, 1], [2, 9]], dtype=torch.int64, device="cuda")
    x = torch.arange(16, dtype=torch.float32, device="cuda").reshape(4, 4)
    out = torch.empty(2, 4, device="cuda")
    call("fmd_pair_aggregate", 0, ptr(x), 4, ptr(bad), 2, 4, ptr(out), ptr(flags), stream())
    torch.cuda.synchronize()
    assert int(flags.item()) & 1
    np.testing.assert_array_equal(out.cpu().numpy(), [[2, 3, 4, 5], [4, 4.5, 5, 5.5]])
    assert _lib.lib().fmd_pair_aggregate(4, ptr(x), 4, ptr(bad), 2, 4, ptr(out), None, None) == 1


def test_admission_on_device():
    from fastmd_b200.pair_aggregate import pair_index_bijection_reason

    ok = torch.tensor([[0, 3], [1, 2]], device="cuda")
    assert pair_index_bijection_reason(ok, 4) is None
    assert pair_index_bijection_reason(torch.tensor([[0, 1], [1, 2]], device="cuda"), 4) == "duplicate_directed_row"
