"""The decomposed indexed-concat SiLU layer on the GPU: the epilogue against the reference's kernels
(golden vectors) and the whole layer against an FP64 evaluation of the concatenated linear.
Tolerances: the epilogue is the reference's FP32 program (expf vs NumPy's exp: 2 ulp), the scattered
gradients sum in CSR order instead of the reference's atomic order (FP32 rounding); the layer's
projections are 3xTF32 (FP32 accuracy)."""
import numpy as np
import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu


def _t(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


@pytest.mark.parametrize("tag", ["cat3", "cat3_sorted_odd", "cat4"])
def test_epilogue_matches_reference_kernels(tag):
    from fastmd_b200.decomposed_indexed_cat_silu_linear import _GatherAddSilu

    z = golden("gather_add_silu")
    g = {k[len(f"gas_{tag}_"):]: z[k] for k in z if k.startswith(f"gas_{tag}_")}
    M, NS, H, cat4, _, bias = (int(v) for v in g["meta"])
    n = 3 if cat4 else 2
    ps = [_t(g[f"p{k}"]).requires_grad_(True) for k in range(n + 1)]
    idx = [_t(g[k]) for k in ("ia", "ib", "ic")[:n]]
    core, gate = _GatherAddSilu.apply(ps[0], _t(g["b"]) if bias else None, n, *ps[1:], *idx)
    np.testing.assert_allclose(core.detach().cpu().numpy(), g["core"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(gate.detach().cpu().numpy(), g["gate"], rtol=1e-6, atol=1e-6)
    grads = torch.autograd.grad([core, gate], ps, [_t(g["gc"]), _t(g["gg"])])
    np.testing.assert_allclose(grads[0].cpu().numpy(), g["gp0"], rtol=1e-6, atol=1e-6)
    for k in range(1, n + 1):
        np.testing.assert_allclose(grads[k].cpu().numpy(), g[f"gp{k}"], rtol=2e-6, atol=2e-6)


@pytest.mark.parametrize("cat4", [False, True])
def test_layer_matches_fp64_concatenated_linear(cat4):
    from fastmd_b200.decomposed_indexed_cat_silu_linear import (decomposed_indexed_cat3_silu_linear,
                                                                 decomposed_indexed_cat4_silu_linear)

    gen = torch.Generator().manual_seed(3)
    rows, NA, NB, D, H = 3000, 400, 250, 128, 64
    A = torch.randn(rows, D, generator=gen)
    X = torch.randn(NA, D, generator=gen)
    B = torch.randn(NB, D, generator=gen)
    ia = torch.randint(0, NA if cat4 else NB, (rows,), generator=gen)
    ib = torch.randint(0, NB, (rows,), generator=gen)
    ic = torch.randint(0, NB, (rows,), generator=gen)
    Ws = [torch.randn(2 * H, D, generator=gen) / 16 for _ in range(4 if cat4 else 3)]
    b = torch.randn(2 * H, generator=gen)
    Ad, Xd, Bd = (v.cuda().requires_grad_(True) for v in (A, X, B))
    if cat4:
        core, gate = decomposed_indexed_cat4_silu_linear(Ad, Xd, ia.cuda(), Bd, ib.cuda(), ic.cuda(),
                                                         tuple(w.cuda() for w in Ws), b.cuda())
        cat = torch.cat([A, X[ia], B[ib], B[ic]], 1).double()
    else:
        core, gate = decomposed_indexed_cat3_silu_linear(Ad, Bd, ia.cuda(), ib.cuda(), tuple(w.cuda() for w in Ws),
                                                         b.cuda())
        cat = torch.cat([A, B[ia], B[ib]], 1).double()
    cat.requires_grad_(True)
    pre = cat @ torch.cat(Ws, 1).double().T + b.double()
    ref_core, ref_gate = torch.nn.functional.silu(pre[:, :H]), torch.nn.functional.silu(pre[:, H:])
    scale = (cat.abs() @ torch.cat(Ws, 1).double().abs().T + b.double().abs()).detach()
    for got, ref, sc in ((core, ref_core, scale[:, :H]), (gate, ref_gate, scale[:, H:])):
        assert ((got.detach().cpu().double() - ref.detach()).abs() / (sc + ref.detach().abs())).max() < 4e-6
    gc = torch.randn(rows, H, generator=gen)
    gg = torch.randn(rows, H, generator=gen)
    gA, *gsrc = torch.autograd.grad([core, gate], [Ad, Xd, Bd] if cat4 else [Ad, Bd], [gc.cuda(), gg.cuda()])
    (gcat,) = torch.autograd.grad([ref_core, ref_gate], [cat], [gc.double(), gg.double()])
    ref_A = gcat[:, :D]
    np.testing.assert_allclose(gA.cpu().numpy(), ref_A.numpy(), rtol=1e-4, atol=2e-5)
    ref_B = torch.zeros(NB, D, dtype=torch.float64)
    if cat4:
        ref_X = torch.zeros(NA, D, dtype=torch.float64).index_add_(0, ia, gcat[:, D:2 * D])
        ref_B.index_add_(0, ib, gcat[:, 2 * D:3 * D]).index_add_(0, ic, gcat[:, 3 * D:])
        np.testing.assert_allclose(gsrc[0].cpu().numpy(), ref_X.numpy(), rtol=1e-4, atol=5e-5)
        np.testing.assert_allclose(gsrc[1].cpu().numpy(), ref_B.numpy(), rtol=1e-4, atol=5e-5)
    else:
        ref_B.index_add_(0, ia, gcat[:, D:2 * D]).index_add_(0, ib, gcat[:, 2 * D:])
        np.testing.assert_allclose(gsrc[0].cpu().numpy(), ref_B.numpy(), rtol=1e-4, atol=5e-5)


def test_guards_decline_like_the_reference():
    from fastmd_b200.decomposed_indexed_cat_silu_linear import decomposed_indexed_cat3_silu_linear

    A = torch.randn(10, 8, device="cuda")
    B = torch.randn(5, 8, device="cuda")
    idx = torch.zeros(10, dtype=torch.int64, device="cuda")
    Ws = tuple(torch.randn(4, 8, device="cuda") for _ in range(3))
    assert decomposed_indexed_cat3_silu_linear(A.t().contiguous().t(), B, idx, idx, Ws) is None  # strided aligned
    assert decomposed_indexed_cat3_silu_linear(A, B, idx, idx, Ws[:2]) is None
    assert decomposed_indexed_cat3_silu_linear(A, B, idx, idx, Ws, bias=torch.randn(2, 2, device="cuda")) is None
    assert decomposed_indexed_cat3_silu_linear(A, B, idx, idx, Ws) is not None
