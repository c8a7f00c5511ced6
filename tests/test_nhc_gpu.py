"""The fused Nose-Hoover-chain kernels against the reference's torch backend (golden) and the oracle."""
import numpy as np
import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu


def _run(tag, cuda, replicas=1, graph=False):
    from fastmd_b200.gpu_nhc import GPUNoseHooverChainNVT, ReplicaNoseHooverChainNVT

    g = golden("nhc")
    n, tchain, tloop, f32, steps = (int(v) for v in g[f"nhc_{tag}_meta"])
    T, dt, tdamp, k = g["nhc_params"]
    q0 = torch.from_numpy(g["nhc_q0"]).to(cuda)
    init = g[f"nhc_{tag}_init"]
    masses, q, p = init[:n], init[n:4 * n].reshape(n, 3), init[4 * n:].reshape(n, 3)
    fdt = torch.float32 if f32 else torch.float64
    kw = dict(temperature_K=T, timestep=dt, tdamp=tdamp, tchain=tchain, tloop=tloop, force_dtype=fdt,
              device=cuda)
    if replicas == 1:
        nhc = GPUNoseHooverChainNVT(masses, q, p, **kw)
    else:
        nhc = ReplicaNoseHooverChainNVT(masses, np.tile(q, (replicas, 1)), np.tile(p, (replicas, 1)),
                                        replicas=replicas, **kw)
    q0r = q0.repeat(replicas, 1)

    def forces(x):
        d = x - q0r
        e = (0.5 * k * (d * d).reshape(replicas, -1).sum(dim=1))
        return (-k * d).to(fdt), e

    f, e = forces(nhc.positions)
    nhc.set_forces(f, e)
    flats = [nhc.state.flat.clone()]
    if graph:
        static = {}
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        g_ = torch.cuda.CUDAGraph()
        snapshot = nhc.snapshot()
        with torch.cuda.stream(stream):
            for _ in range(2):  # warm-up
                x = nhc.step_pre_force()
                f, e = forces(x)
                nhc.step_post_force(f, e)
        torch.cuda.current_stream().wait_stream(stream)
        nhc.load_snapshot(snapshot)
        with torch.cuda.graph(g_):
            x = nhc.step_pre_force()
            f, e = forces(x)
            nhc.step_post_force(f, e)
        for _ in range(steps):
            g_.replay()
            flats.append(nhc.state.flat.clone())
    else:
        for _ in range(steps):
            x = nhc.step_pre_force()
            f, e = forces(x)
            nhc.step_post_force(f, e)
            flats.append(nhc.state.flat.clone())
    return nhc, torch.stack(flats).cpu().numpy(), g[f"nhc_{tag}_flat"], n, tchain


def _layout_single(flat, n, M, R, r):
    """Replica r's [q|p|F|eta|p_eta|E] from the R-replica layout."""
    n3 = 3 * n
    q = flat[:, r * n3:(r + 1) * n3]
    p = flat[:, R * n3 + r * n3:R * n3 + (r + 1) * n3]
    f = flat[:, 2 * R * n3 + r * n3:2 * R * n3 + (r + 1) * n3]
    base = 3 * R * n3
    eta = flat[:, base + r * M:base + (r + 1) * M]
    pe = flat[:, base + R * M + r * M:base + R * M + (r + 1) * M]
    e = flat[:, base + 2 * R * M + r:base + 2 * R * M + r + 1]
    return np.concatenate([q, p, f, eta, pe, e], axis=1)


def _max_rel(a, b):
    scale = np.maximum(np.abs(b).max(axis=0, keepdims=True), 1e-30)
    return float(np.max(np.abs(a - b) / scale))


@pytest.mark.parametrize("tag", ["f64_m3_l1", "f32_m3_l1", "f64_m1_l1", "f64_m5_l2"])
def test_nhc_matches_reference_trajectory(cuda, tag):
    _, mine, ref, n, M = _run(tag, cuda)
    assert mine.shape == ref.shape
    assert _max_rel(mine, ref) < 1e-12


def test_replicas_bitwise_equal_single_system(cuda):
    _, single, _, n, M = _run("f64_m3_l1", cuda)
    _, rep, _, _, _ = _run("f64_m3_l1", cuda, replicas=4)
    for r in range(4):
        assert np.array_equal(_layout_single(rep, n, M, 4, r), single)


def test_graph_replay_bitwise_equal_eager(cuda):
    _, eager, _, _, _ = _run("f32_m3_l1", cuda)
    _, replay, _, _, _ = _run("f32_m3_l1", cuda, graph=True)
    assert np.array_equal(eager, replay)


def test_backup_restore_and_observables(cuda):
    nhc, _, _, n, M = _run("f64_m3_l1", cuda)
    nhc.backup()
    before = nhc.state.flat.clone()
    nhc.step_pre_force()
    nhc.restore()
    assert torch.equal(before, nhc.state.flat)
    ke = float(nhc.kinetic_energy())
    p = nhc.momenta.cpu().numpy()
    m = nhc.masses.cpu().numpy()
    assert abs(ke - 0.5 * np.sum(p * p / m)) < 1e-12 * abs(ke)
    assert np.isfinite(float(nhc.conserved_energy()))


def test_positions32_follow_the_drift(cuda):
    nhc, _, _, _, _ = _run("f64_m3_l1", cuda)
    assert torch.equal(nhc.positions32, nhc.positions.float())


@pytest.mark.parametrize("tag", ["f32", "f64"])
@pytest.mark.parametrize("replicas", [1, 3])
def test_fused_post_pre_half_equals_the_two_halves(cuda, tag, replicas):
    """fmd_nhc_post_pre_force (the two halves between two force calls in one launch) leaves the state,
    the float32 positions and the cached forces and energies bitwise equal to post-force then pre-force."""
    from fastmd_b200.gpu_nhc import GPUNoseHooverChainNVT, ReplicaNoseHooverChainNVT

    rng = np.random.default_rng(3)
    n = 135
    masses = rng.uniform(100.0, 140.0, n)
    q = rng.uniform(0.0, 18.6, (replicas * n, 3))
    p = rng.normal(0.0, 2.0, (replicas * n, 3))
    fdt = torch.float32 if tag == "f32" else torch.float64
    kw = dict(temperature_K=500.0, timestep=0.0245, tdamp=2.45, tchain=3, tloop=1, force_dtype=fdt, device=cuda)
    make = (lambda: GPUNoseHooverChainNVT(masses, q, p, **kw)) if replicas == 1 else (
        lambda: ReplicaNoseHooverChainNVT(masses, q, p, replicas=replicas, **kw))
    a, b = make(), make()
    for nhc in (a, b):
        nhc.set_forces(torch.zeros((replicas * n, 3), dtype=fdt, device=cuda), torch.zeros(replicas, device=cuda,
                                                                                             dtype=torch.float64))
        nhc.step_pre_force()
    for step in range(4):
        f = torch.from_numpy(rng.normal(0.0, 1.0, (replicas * n, 3))).to(cuda, fdt)
        e = torch.from_numpy(rng.normal(-5.0, 1.0, replicas)).to(cuda)
        a.step_post_force(f, e)
        a.step_pre_force()
        b.step_post_pre_force(f, e)
        torch.cuda.synchronize()
        assert torch.equal(a.state.flat, b.state.flat), step
        assert torch.equal(a.positions32, b.positions32), step


@pytest.mark.parametrize("n", [1500, 5000, 10000])
def test_large_replica_clusters_match_the_oracle(cuda, n):
    """A replica of more than 4,096 degrees of freedom runs on a thread-block cluster (4 or 8 CTAs, the
    kinetic-energy sums combined across the cluster in rank order): 10 steps under harmonic forces
    against the FP64 oracle NHC (1e-12 of each block's scale), two replicas as a union bitwise equal to
    each run alone, and the fused post/pre half bitwise equal to the two halves."""
    from fastmd_b200.gpu_nhc import GPUNoseHooverChainNVT, ReplicaNoseHooverChainNVT
    from oracle.nhc import NHC

    rng = np.random.default_rng(n)
    masses = rng.uniform(100.0, 140.0, n)
    q0 = rng.uniform(0.0, 40.0, (n, 3))
    p0 = rng.normal(0.0, 2.0, (n, 3))
    k = 0.7
    kw = dict(temperature_K=500.0, timestep=0.0245, tdamp=2.45, tchain=3, tloop=1)

    def forces(x, ref):
        d = x - ref
        return -k * d, 0.5 * k * float((d * d).sum())

    ref = NHC(masses, q0, p0, np.zeros((n, 3)), **kw)
    gpu = GPUNoseHooverChainNVT(masses, q0, p0, force_dtype=torch.float64, device=cuda, **kw)
    q0d = torch.from_numpy(q0).to(cuda)
    gpu.set_forces(torch.zeros((n, 3), dtype=torch.float64, device=cuda),
                   torch.zeros(1, dtype=torch.float64, device=cuda))
    for _ in range(10):
        x = ref.pre_force()
        f, e = forces(x, q0)
        ref.post_force(f, e)
        xg = gpu.step_pre_force()
        fg = -k * (xg - q0d)
        gpu.step_post_force(fg, (0.5 * k * ((xg - q0d) ** 2).sum()).reshape(1))
    flat = gpu.state.flat.cpu().numpy()
    want = ref.flat()
    n3 = 3 * n
    for lo, hi in ((0, n3), (n3, 2 * n3), (2 * n3, 3 * n3), (3 * n3, 3 * n3 + 6)):
        scale = max(np.abs(want[lo:hi]).max(), 1e-30)
        assert np.abs(flat[lo:hi] - want[lo:hi]).max() <= 1e-12 * scale, (lo, hi)

    # two replicas as one union: each bitwise equal to its run alone
    p1 = rng.normal(0.0, 2.0, (n, 3))
    union = ReplicaNoseHooverChainNVT(masses, np.concatenate([q0, q0]), np.concatenate([p0, p1]), replicas=2,
                                      force_dtype=torch.float64, device=cuda, **kw)
    alone = [GPUNoseHooverChainNVT(masses, q0, pp, force_dtype=torch.float64, device=cuda, **kw) for pp in (p0, p1)]
    fz = torch.zeros((n, 3), dtype=torch.float64, device=cuda)
    ez = torch.zeros(1, dtype=torch.float64, device=cuda)
    union.set_forces(torch.cat([fz, fz]), torch.zeros(2, dtype=torch.float64, device=cuda))
    for a in alone:
        a.set_forces(fz, ez)
    for step in range(3):
        fu = torch.from_numpy(rng.normal(0.0, 1.0, (2 * n, 3))).to(cuda)
        union.step_pre_force()
        union.step_post_force(fu, torch.ones(2, dtype=torch.float64, device=cuda))
        for r, a in enumerate(alone):
            a.step_pre_force()
            a.step_post_force(fu[r * n:(r + 1) * n].contiguous(), torch.ones(1, dtype=torch.float64, device=cuda))
    torch.cuda.synchronize()
    uq = union.state.q.reshape(-1)
    for r, a in enumerate(alone):
        assert torch.equal(uq[r * n3:(r + 1) * n3], a.state.q.reshape(-1))

    # the fused post/pre half
    b = GPUNoseHooverChainNVT(masses, q0, p0, force_dtype=torch.float64, device=cuda, **kw)
    c = GPUNoseHooverChainNVT(masses, q0, p0, force_dtype=torch.float64, device=cuda, **kw)
    for s_ in (b, c):
        s_.set_forces(fz, ez)
        s_.step_pre_force()
    for step in range(3):
        f = torch.from_numpy(rng.normal(0.0, 1.0, (n, 3))).to(cuda)
        b.step_post_force(f, ez)
        b.step_pre_force()
        c.step_post_pre_force(f, ez)
        torch.cuda.synchronize()
        assert torch.equal(b.state.flat, c.state.flat), step
