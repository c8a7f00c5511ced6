"""The tcgen05 3xTF32 wide GEMM (fmd_gemm_tf32x3, fmd_tf32_split) against the CPU oracle.

Tolerance: the kernel differs from the exact 3xTF32 value (oracle/wide_gemm.py) by the FP32 rounding of
its accumulations inside one 64-wide K chunk (24 tensor-core additions), the FP32 sum of the chunks
and the TF32 read of lo: |y - oracle| <= 4e-6 * sum_k |x||w| (+ |bias| + |c|).
"""
import numpy as np
import pytest
import torch

from oracle import wide_gemm as ow

pytestmark = pytest.mark.gpu
TOL = 4e-6


def _data(m, n, k, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g) * scale
    w = torch.randn(n, k, generator=g) / np.sqrt(k)
    b = torch.randn(n, generator=g)
    return x, w, b


def _check(y, x, w, bias=None, c=None, act=0, tol=TOL):
    xn, wn = x.numpy(), w.numpy()
    bn = None if bias is None else bias.numpy()
    cn = None if c is None else c.numpy()
    ref = ow.gemm_3xtf32(xn, wn, bn, cn)
    scale = ow.error_scale(xn, wn, bn, cn)
    got = y.detach().cpu().double().numpy()
    if act == 1:
        ref = ref / (1.0 + np.exp(-ref))
        # SiLU's slope is within [-0.1, 1.1]; its FP32 evaluation adds a few ulps of the output
        scale = 1.1 * scale + np.abs(ref)
    err = np.abs(got - ref) / scale
    assert np.all(np.isfinite(got))
    assert err.max() < tol, (err.max(), np.unravel_index(err.argmax(), err.shape))


def test_tf32_split_bitwise():
    from fastmd_b200 import wide_gemm

    w = torch.randn(200, 72) * 10
    dev = w.cuda()
    for transposed in (False, True):
        sp = wide_gemm._split(dev, transposed)
        hi, lo = ow.split(w.numpy().T.copy() if transposed else w.numpy())
        np.testing.assert_array_equal(sp.hi.cpu().numpy(), hi)
        np.testing.assert_array_equal(sp.lo.cpu().numpy(), lo)
    # cached per weight version, rebuilt after an in-place update
    assert wide_gemm._split(dev, False) is wide_gemm._split(dev, False)
    dev.mul_(2.0)
    np.testing.assert_array_equal(wide_gemm._split(dev, False).hi.cpu().numpy(), ow.split(w.numpy() * 2)[0])


@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (5, 7, 3), (129, 64, 64), (300, 128, 256), (1000, 256, 264),
                                   (257, 264, 256), (4097, 96, 100), (700, 200, 1000),
                                   # narrow tiles (n <= 64: 64-column accumulators, five A buffers, n-row w boxes)
                                   (40000, 64, 512), (2000, 33, 100), (700, 16, 40), (3000, 48, 64)])
def test_linear_matches_oracle(m, n, k):
    from fastmd_b200 import wide_gemm

    x, w, b = _data(m, n, k, seed=m + n + k)
    y = wide_gemm.linear(x.cuda(), w.cuda(), b.cuda())
    torch.cuda.synchronize()
    _check(y, x, w, b)


def test_residual_silu_accumulate_and_ieee():
    from fastmd_b200 import _lib, wide_gemm
    from fastmd_b200._lib import call, ptr

    m, n, k = 515, 256, 264
    x, w, b = _data(m, n, k, seed=7)
    c = torch.randn(m, n, generator=torch.Generator().manual_seed(8))
    xd, wd, bd, cd = x.cuda(), w.cuda(), b.cuda(), c.cuda()
    _check(wide_gemm.linear(xd, wd, bd, act=1), x, w, b, act=1)
    # the residual: y = x w^T + b + c, in place into c (matmul's accumulate form on the forward operand)
    sp = wide_gemm._split(wd, False)
    y = cd.clone()
    s = _lib.stream()
    call("fmd_gemm_tf32x3", ptr(xd), k, ptr(sp.hi), ptr(sp.lo), k, ptr(bd), ptr(y), n, ptr(y), n, m, n, k, 0, 0,
         None, s)
    _check(y, x, w, b, c)
    # accumulate: y += act(...)
    y2 = cd.clone()
    call("fmd_gemm_tf32x3", ptr(xd), k, ptr(sp.hi), ptr(sp.lo), k, ptr(bd), None, 0, ptr(y2), n, m, n, k, 1, 1,
         None, s)
    ref = torch.nn.functional.silu(torch.from_numpy(ow.gemm_3xtf32(x.numpy(), w.numpy(), b.numpy()))) + c.double()
    scale = 1.1 * torch.from_numpy(ow.error_scale(x.numpy(), w.numpy(), b.numpy())) + ref.abs()
    assert ((y2.cpu().double() - ref).abs() / scale).max() < TOL
    # an output row stride the TMA cannot take (257 floats): the direct-store epilogue
    out = torch.empty(m, n + 1, device="cuda")[:, :n]
    wide_gemm.linear_into(out, xd, wd, bd)
    _check(out, x, w, b)
    # the IEEE parity path through the same surface
    yi = wide_gemm.linear(xd, wd, bd, precision="ieee")
    _check(yi, x, w, b, tol=2e-6)


def test_matmul_input_gradient_and_autograd():
    from fastmd_b200 import wide_gemm

    m, n, k = 333, 256, 264
    _, w, _ = _data(m, n, k, seed=11)
    g = torch.randn(m, n, generator=torch.Generator().manual_seed(10))
    gd, wd = g.cuda(), w.cuda()
    # dX = dY @ W : the oracle of grad [m, n] @ w [n, k] is gemm_3xtf32(grad, w^T)
    wt = w.t().contiguous()
    _check(wide_gemm.matmul(gd, wd), g, wt)
    c = torch.randn(m, k, generator=torch.Generator().manual_seed(12))
    cd = c.cuda()
    out = wide_gemm.matmul(gd, wd, c=cd, accumulate=True)
    assert out.data_ptr() == cd.data_ptr()
    _check(out, g, wt, c=c)
    # autograd: forward linear, backward through matmul
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(13))
    xd = x.cuda().requires_grad_(True)
    y = wide_gemm.linear(xd, wd)
    gy = torch.randn(m, n, generator=torch.Generator().manual_seed(14))
    y.backward(gy.cuda())
    _check(xd.grad, gy, wt)


def test_row_results_do_not_depend_on_rows_or_tiles():
    """A row's output is a function of its own inputs only: bitwise equal under any row count/offset."""
    from fastmd_b200 import wide_gemm

    x, w, b = _data(1000, 256, 264, seed=21)
    xd, wd, bd = x.cuda(), w.cuda(), b.cuda()
    full = wide_gemm.linear(xd, wd, bd)
    part = wide_gemm.linear(xd[300:377].contiguous(), wd, bd)
    assert torch.equal(full[300:377], part)
    again = wide_gemm.linear(xd, wd, bd)
    assert torch.equal(full, again)


def test_large_rows_sampled():
    """A config-2-like shape (K 264 -> N 256) at 300k rows: sampled rows against the oracle, and the
    unaligned row stride of a strided view handled by the wrapper (a TMA-legal copy)."""
    from fastmd_b200 import wide_gemm

    m, n, k = 300_000, 256, 264
    g = torch.Generator(device="cuda").manual_seed(5)
    xd = torch.randn(m, k, device="cuda", generator=g)
    wd = torch.randn(n, k, device="cuda", generator=g) / 16
    bd = torch.randn(n, device="cuda", generator=g)
    y = wide_gemm.linear(xd, wd, bd, act=1)
    rows = torch.randint(0, m, (512,), generator=torch.Generator().manual_seed(6))
    rows = torch.cat([rows, torch.tensor([0, m - 1])])
    _check(y[rows.cuda()], xd[rows.cuda()].cpu(), wd.cpu(), bd.cpu(), act=1)
    # a view whose row stride (265 floats) breaks the 16-byte TMA rule
    base = torch.randn(1000, k + 1, device="cuda", generator=g)
    view = base[:, 1:]
    _check(wide_gemm.linear(view, wd, bd), view.cpu().contiguous(), wd.cpu(), bd.cpu())


@pytest.mark.parametrize("m,n,k", [(1000, 64, 64), (333, 256, 264), (77, 5, 3)])
def test_input_silu_and_silu_grad_modes(m, n, k):
    """FMD_ACT_INPUT_SILU (the operand enters as silu(x)) and FMD_ACT_SILU_GRAD (y = (x w^T + b) silu'(c),
    in place over c) against the oracle: the layers of an MLP chained on pre-activations and their
    backward. silu and silu' run on the hardware exp2 / divide: a few ulp of the operand or the gate."""
    from fastmd_b200 import _lib, wide_gemm
    from fastmd_b200._lib import call, ptr

    x, w, b = _data(m, n, k, seed=m + 3 * n + k)
    ldx = (k + 3) // 4 * 4  # TMA: a row stride of whole 16-byte units
    xd = torch.zeros(m, ldx, device="cuda")
    xd[:, :k] = x.cuda()
    wd, bd = w.cuda(), b.cuda()
    sp = wide_gemm._split(wd, False)
    ldw = sp.hi.stride(0)
    s = _lib.stream()
    # input SiLU, SiLU output as well: y = silu(silu(x) w^T + b)
    y = torch.empty(m, n, device="cuda")
    call("fmd_gemm_tf32x3", ptr(xd), ldx, ptr(sp.hi), ptr(sp.lo), ldw, ptr(bd), None, 0, ptr(y), n, m, n, k, 1 | 16,
         0, None, s)
    sx = torch.nn.functional.silu(x.double()).float()
    _check(y, sx, w, b, act=1, tol=2e-5)
    # silu' gate, in place over the pre-activation c
    c = torch.randn(m, n, generator=torch.Generator().manual_seed(99)) * 3
    cd = c.cuda()
    call("fmd_gemm_tf32x3", ptr(xd), ldx, ptr(sp.hi), ptr(sp.lo), ldw, ptr(bd), ptr(cd), n, ptr(cd), n, m, n, k, 2,
         0, None, s)
    torch.cuda.synchronize()
    sig = torch.sigmoid(c.double())
    gate = (sig * (1 + c.double() * (1 - sig))).numpy()
    acc = ow.gemm_3xtf32(x.numpy(), w.numpy(), b.numpy())
    # the product's error scaled by the gate, plus the gate's own absolute error (hardware exp2 and
    # divide: s to a few ulp, then 1 - s and c (1 - s) for |c| <= 12: below 1e-5)
    bound = TOL * ow.error_scale(x.numpy(), w.numpy(), b.numpy()) * np.abs(gate) + 1e-5 * np.abs(acc) + 1e-12
    err = np.abs(cd.cpu().double().numpy() - acc * gate) / bound
    assert err.max() < 1.0, err.max()
    # mode 2 without c is an argument error
    lib = _lib.lib()
    assert lib.fmd_gemm_tf32x3(ptr(xd), ldx, ptr(sp.hi), ptr(sp.lo), ldw, None, None, 0, ptr(y), n, m, n, k, 2, 0,
                               None, s) == 1


@pytest.mark.parametrize("shapes", [
    [(5000, 128, 128, 0), (15000, 64, 64, 0), (25000, 32, 32, 0)],        # a NequIP block's per-l linears
    [(5000, 224, 128, 0), (15000, 64, 384, 0), (25000, 32, 352, 0)],      # their input gradients
    [(3000, 64, 64, 16), (3000, 64, 64, 16), (777, 48, 100, 0), (129, 8, 320, 0)],  # narrow only, 4 problems
    [(0, 64, 64, 0), (1000, 256, 264, 1)],                                # an empty problem skipped
])
def test_grouped_problems_equal_single_calls(shapes):
    """fmd_gemm_tf32x3_grouped: each problem's output equals its own fmd_gemm_tf32x3 call bit for bit,
    whether the group runs as narrow (every n <= 64) or wide tiles."""
    from fastmd_b200 import wide_gemm

    g = torch.Generator(device="cuda").manual_seed(len(shapes))
    problems, singles = [], []
    for m, n, k, act in shapes:
        ld = (k + 3) // 4 * 4
        a = torch.randn(m, ld, device="cuda", generator=g)[:, :k]
        w = torch.randn(n, k, device="cuda", generator=g) / k ** 0.5
        b = torch.randn(n, device="cuda", generator=g)
        problems.append({"a": a, "weight": w, "bias": b, "act": act})
        singles.append(wide_gemm._launch(a, w, False, "tf32x3", b, act=act))
    outs = wide_gemm.grouped(problems)
    torch.cuda.synchronize()
    for y, ref in zip(outs, singles):
        assert torch.equal(y, ref)


def test_matches_the_reference_kernel_outputs():
    """fmd_gemm_tf32x3 against the outputs of the reference's own 3xTF32 kernels on the same inputs (the
    golden fixture: fastmd/engine/kernels/triton_wide_gemm.py under the Triton interpreter, FP32 dots): the
    forward with bias, the accumulate form (+ c), the input-gradient orientation (dX = dY W into c), a
    64-wide tile and K = 448. Bar: the kernel's own bound against the exact 3xTF32 value plus the
    fixture's FP32 rounding (below 2e-7 of the same scale)."""
    import sys
    from pathlib import Path

    from fastmd_b200 import _lib, wide_gemm
    from fastmd_b200._lib import call, ptr

    here = Path(__file__).resolve().parent / "golden"
    sys.path.insert(0, str(here))
    from inputs import WIDE_GEMM_CASES, wide_gemm_inputs

    golden = np.load(here / "wide_gemm.npz")
    s = _lib.stream()
    for i, (tag, (m, k, n, transposed, has_bias, has_c)) in enumerate(WIDE_GEMM_CASES.items()):
        a, w, bias, c = wide_gemm_inputs(i, m, k, n, transposed, has_bias, has_c)
        ad, wd = torch.from_numpy(a).cuda(), torch.from_numpy(w).cuda()
        bd = torch.from_numpy(bias).cuda() if has_bias else None
        cd = torch.from_numpy(c).cuda() if has_c else None
        sp = wide_gemm._split(wd, transposed)  # the K-major [n, k] pair of B
        y = torch.empty(m, n, device="cuda")
        call("fmd_gemm_tf32x3", ptr(ad), k, ptr(sp.hi), ptr(sp.lo), k, ptr(bd) if has_bias else None,
             ptr(cd) if has_c else None, n if has_c else 0, ptr(y), n, m, n, k, 0, 0, None, s)
        torch.cuda.synchronize()
        wk = np.ascontiguousarray(w.T if transposed else w)
        scale = ow.error_scale(a, wk, bias=bias, c=c)
        err = np.abs(y.cpu().double().numpy() - golden[f"wg_{tag}_y"].astype(np.float64)) / scale
        assert err.max() < TOL + 2e-7, (tag, err.max())
