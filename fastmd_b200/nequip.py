"""NequIP-architecture (SevenNet-0-style) potential on this build's kernels: BASELINE config 3's model.

The reference wraps upstream SevenNet (fastmd/models/sevennet.py, ``sevenn==0.13.0``: an E(3)-equivariant
NequIP network); this is the same architecture family with random weights, as config 3 asks: species
embedding to 128x0e; 5 interaction blocks on node features 128x0e + 64x1e + 32x2e (no parity), each a
self-connection (an element-dependent linear per l), a linear per l, a tensor-product convolution
over the neighbours weighted per edge by a radial network (8 Bessel functions with a polynomial
envelope -> 64 -> 64 -> 960 path weights, SiLU, no bias) over the 15 couplings l1 (x) l2 -> l3 of the
spherical harmonics up to l = 2, normalised by the average neighbour count, a second linear per l
and a gated nonlinearity (SiLU on the scalars, sigmoid gates on l = 1, 2), plus the self-connection;
then a scalar readout 128 -> 64 -> 1, scaled and shifted, summed per system in FP64. Forces are minus
the position gradient, through the autograd graph of this build's kernels: the edge basis and its
backward (``fmd_nequip_edge_basis``), the convolution and its backward (``fmd_nequip_conv``), the
linears on the tcgen05 wide GEMM (``precision="tf32x3"``) or its IEEE path (``"ieee"``), the position
gradient summed over the receiver and sender CSRs (``fmd_csr_segment_sum``). Element indices are
atomic number - 1 (89 elements). The padded rows of an exact-rc build (``PaddingRule("exact_rc_loops")``,
fastmd/models/sevennet.py:16-22) read the override vector, which the envelope maps to zero.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
from torch import Tensor
from torch.autograd import Function

from . import _lib, ops, wide_gemm
from ._lib import call, ptr, stream
from .graph import _host_cell

MULT = (128, 64, 32)
DIM = (1, 3, 5)
PATHS = [(l1, l2, l3) for l1 in range(3) for l2 in range(3) for l3 in range(3) if abs(l1 - l2) <= l3 <= l1 + l2]
X_WIDTH = sum(m * d for m, d in zip(MULT, DIM))          # 480
M_MULT = tuple(sum(MULT[p[0]] for p in PATHS if p[2] == l) for l in range(3))  # (224, 384, 352)
W_WIDTH = sum(MULT[p[0]] for p in PATHS)                  # 960


@dataclass(frozen=True)
class NequIPConfig:
    num_layers: int = 5
    r_max: float = 5.0
    num_bessel: int = 8
    poly_p: int = 6
    radial_hidden: int = 64
    avg_num_neighbors: float = 11.0
    n_elements: int = 89
    readout_hidden: int = 64
    scale: float = 1.0
    shift: float = 0.0


def init_weights(config: NequIPConfig, seed: int = 1) -> dict[str, np.ndarray]:
    """Random float32 weights (normal, scaled by 1 / sqrt(fan-in))."""
    rng = np.random.default_rng(seed)

    def normal(*shape, fan_in):
        return (rng.standard_normal(shape) / np.sqrt(fan_in)).astype(np.float32)

    w = {"embed": rng.standard_normal((config.n_elements, MULT[0])).astype(np.float32)}
    H = config.radial_hidden
    for L in range(config.num_layers):
        for l in range(3):
            w[f"L{L}.sc{l}"] = normal(config.n_elements, MULT[l], MULT[l], fan_in=MULT[l])
            w[f"L{L}.lin1_{l}"] = normal(MULT[l], MULT[l], fan_in=MULT[l])
        w[f"L{L}.rad1"] = normal(H, config.num_bessel, fan_in=config.num_bessel)
        w[f"L{L}.rad2"] = normal(H, H, fan_in=H)
        w[f"L{L}.rad3"] = normal(W_WIDTH, H, fan_in=H)
        w[f"L{L}.lin2_0"] = normal(M_MULT[0], MULT[0] + MULT[1] + MULT[2], fan_in=M_MULT[0])
        w[f"L{L}.lin2_1"] = normal(M_MULT[1], MULT[1], fan_in=M_MULT[1])
        w[f"L{L}.lin2_2"] = normal(M_MULT[2], MULT[2], fan_in=M_MULT[2])
    w["readout1"] = normal(config.readout_hidden, MULT[0], fan_in=MULT[0])
    w["readout2"] = normal(1, config.readout_hidden, fan_in=config.readout_hidden)
    return w


def coupling_table() -> np.ndarray:
    """The 615 dense coupling constants of the 15 paths (in path order), float32."""
    from ._coupling import clebsch_gordan

    return np.concatenate([clebsch_gordan(*p).reshape(-1) for p in PATHS]).astype(np.float32)


class _EdgeBasis(Function):
    """(Y [E, 9], B [E, n_basis]) of the edges; the backward returns the position gradient."""

    @staticmethod
    def forward(ctx, pos, model, batch):
        E = int(batch.edge_index.shape[0])
        dev = pos.device
        c = model.config
        Y = torch.empty(E, 9, device=dev)
        B = torch.empty(E, c.num_bessel, device=dev)
        geo = torch.empty(E, 4, device=dev)
        cell_ptr = model.cell_ptr(batch)
        override = getattr(batch, "edge_vec_override", None)
        call("fmd_nequip_edge_basis", ptr(pos), cell_ptr, ptr(batch.edge_index), ptr(batch.edge_image), ptr(override),
             ptr(batch.n_edges) if override is not None else None, E, c.r_max, c.num_bessel, c.poly_p, ptr(Y), ptr(B),
             ptr(geo), stream(dev))
        ctx.model, ctx.batch = model, batch
        ctx.save_for_backward(geo)
        return Y, B

    @staticmethod
    def backward(ctx, dY, dB):
        (geo,) = ctx.saved_tensors
        batch, c = ctx.batch, ctx.model.config
        E, N = int(geo.shape[0]), batch.n_real
        g = torch.empty(E, 3, device=geo.device)
        override = getattr(batch, "edge_vec_override", None)
        call("fmd_nequip_edge_basis_bwd", ptr(geo), ptr(dY.contiguous()), ptr(dB.contiguous()), ptr(override),
             ptr(batch.n_edges) if override is not None else None, E, c.r_max, c.num_bessel, c.poly_p, ptr(g),
             stream(geo.device))
        # dE/dpos_a = sum over sent edges (a = neighbour) - sum over received edges (a = centre)
        n_pos = batch.positions.shape[0]
        recv = ops.csr_segment_sum(g, batch.edge_index[:, 0].long(), N, None, batch.recv_off[:N + 1], True)
        send = ops.csr_segment_sum(g, batch.edge_index[:, 1].long(), N, batch.send_perm.long(),
                                   batch.send_off[:N + 1])
        grad = torch.zeros(n_pos, 3, device=geo.device)
        grad[:N] = send - recv
        return grad, None, None


def _planes(flat: Tensor, n: int, mults) -> tuple[Tensor, ...]:
    """The l planes of a planar buffer as [n (2l + 1), mult] matrices (views)."""
    out, off = [], 0
    for m, d in zip(mults, DIM):
        out.append(flat[off:off + n * m * d].view(n * d, m))
        off += n * m * d
    return tuple(out)


class _Conv(Function):
    """Messages (three planes [N, 224], [3N, 384], [5N, 352]) of the node features x (the planar buffer
    of 480 N floats); the backward returns the gradients of x, Y and W."""

    @staticmethod
    def forward(ctx, x, Y, W, model, batch):
        N = batch.n_real
        m = torch.empty(N * sum(M_MULT[l] * DIM[l] for l in range(3)), device=x.device)
        call("fmd_nequip_conv", ptr(x), ptr(Y), ptr(W), ptr(model.cg), ptr(batch.edge_index), ptr(batch.recv_off), N,
             1.0 / model.config.avg_num_neighbors, ptr(m), stream(x.device))
        ctx.save_for_backward(x, Y, W)
        ctx.model, ctx.batch = model, batch
        return _planes(m, N, M_MULT)

    @staticmethod
    def backward(ctx, *dm):
        x, Y, W = ctx.saved_tensors
        model, batch = ctx.model, ctx.batch
        N = batch.n_real
        dm = torch.cat([(g if g is not None else torch.zeros(N * M_MULT[l] * DIM[l], device=x.device)).reshape(-1)
                        for l, g in enumerate(dm)])
        gx, gW, gY = torch.empty_like(x), torch.empty_like(W), torch.empty_like(Y)
        call("fmd_nequip_conv_bwd", ptr(x), ptr(Y), ptr(W), ptr(model.cg), ptr(batch.edge_index), ptr(batch.recv_off),
             ptr(batch.send_off), ptr(batch.send_perm), N, 1.0 / model.config.avg_num_neighbors, ptr(dm), ptr(gx),
             ptr(gW), ptr(gY), stream(x.device))
        return gx, gY, gW, None, None


class _SelfConnection(Function):
    """The element-dependent linear of the three feature planes (``fmd_nequip_self_connection``); its
    input gradient is the same kernel on the transposed weights ``t0, t1, t2`` (frozen; kept as copies
    so that both directions read a weight row across the warp's consecutive output channels)."""

    @staticmethod
    def forward(ctx, x0, x1, x2, elem, w0, w1, w2, t0, t1, t2):
        n = x0.shape[0]
        xs = [x0.contiguous(), x1.contiguous(), x2.contiguous()]
        out = [torch.empty_like(t) for t in xs]
        call("fmd_nequip_self_connection", ptr(xs[0]), ptr(xs[1]), ptr(xs[2]), ptr(elem), ptr(w0), ptr(w1), ptr(w2), n,
             0, ptr(out[0]), ptr(out[1]), ptr(out[2]), stream(x0.device))
        ctx.save_for_backward(elem, t0, t1, t2)
        return tuple(out)

    @staticmethod
    def backward(ctx, g0, g1, g2):
        elem, t0, t1, t2 = ctx.saved_tensors
        gs = [g.contiguous() for g in (g0, g1, g2)]
        dx = [torch.empty_like(g) for g in gs]
        call("fmd_nequip_self_connection", ptr(gs[0]), ptr(gs[1]), ptr(gs[2]), ptr(elem), ptr(t0), ptr(t1), ptr(t2),
             gs[0].shape[0], 0, ptr(dx[0]), ptr(dx[1]), ptr(dx[2]), stream(gs[0].device))
        return dx[0], dx[1], dx[2], None, None, None, None, None, None, None


class _Gate(Function):
    """(x0 [N, 128], x1 [3N, 64], x2 [5N, 32]) = the gated nonlinearity of the second linear's outputs
    (o0 [N, 224], o1 [3N, 64], o2 [5N, 32]) plus the self-connection planes sc (``fmd_nequip_gate``)."""

    @staticmethod
    def forward(ctx, o0, o1, o2, sc0, sc1, sc2):
        n = o0.shape[0]
        o0, o1, o2 = o0.contiguous(), o1.contiguous(), o2.contiguous()
        x = [torch.empty(n * DIM[l], MULT[l], device=o0.device) for l in range(3)]
        call("fmd_nequip_gate", ptr(o0), ptr(o1), ptr(o2), ptr(sc0.contiguous()), ptr(sc1.contiguous()),
             ptr(sc2.contiguous()), n, ptr(x[0]), ptr(x[1]), ptr(x[2]), stream(o0.device))
        ctx.save_for_backward(o0, o1, o2)
        return tuple(x)

    @staticmethod
    def backward(ctx, dx0, dx1, dx2):
        o0, o1, o2 = ctx.saved_tensors
        n = o0.shape[0]
        dx = [g.contiguous() if g is not None else torch.zeros(n * DIM[l], MULT[l], device=o0.device)
              for l, g in enumerate((dx0, dx1, dx2))]
        do = [torch.empty_like(o0), torch.empty_like(o1), torch.empty_like(o2)]
        call("fmd_nequip_gate_bwd", ptr(o0), ptr(o1), ptr(o2), ptr(dx[0]), ptr(dx[1]), ptr(dx[2]), n, ptr(do[0]),
             ptr(do[1]), ptr(do[2]), stream(o0.device))
        return do[0], do[1], do[2], dx[0], dx[1], dx[2]


def gate(o0: Tensor, o1: Tensor, o2: Tensor, sc0: Tensor, sc1: Tensor, sc2: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    """The block's gated nonlinearity plus self-connection on the device (differentiable)."""
    return _Gate.apply(o0, o1, o2, sc0, sc1, sc2)


class NequIPModel:
    """The config-3 potential on the device. ``energy_forces(batch)`` -> (energy [1] fp64, forces [N, 3])
    for a ``GraphBatch`` of one system (receiver and sender CSRs of its edges)."""

    def __init__(self, config: NequIPConfig | None = None, weights: dict | None = None, *, seed: int = 1,
                 device="cuda", precision: str = "tf32x3") -> None:
        self.config = config or NequIPConfig()
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise _lib.FastMDLibraryError("the NequIP kernels run on CUDA devices only")
        host = weights if weights is not None else init_weights(self.config, seed)
        self.host_weights = host
        self.w = {k: torch.as_tensor(v, dtype=torch.float32, device=self.device) for k, v in host.items()}
        # the matrices the GEMM reads as [out, in]
        self.lin = {k: v.t().contiguous() for k, v in self.w.items() if ".lin" in k}
        # the layers' first radial layers stacked [layers * hidden, n_basis]: one GEMM for all layers
        self.rad1_all = torch.cat([self.w[f"L{L}.rad1"] for L in range(self.config.num_layers)], 0).contiguous()
        # self-connection weights [elements, out, in] for the input gradient
        self.sc_t = {k: v.transpose(1, 2).contiguous() for k, v in self.w.items() if ".sc" in k}
        self.precision = precision
        self.cg = torch.as_tensor(coupling_table(), device=self.device)

    # ------------------------------------------------------------ per-system state (no host work per call)
    def prepare(self, batch):
        """The element rows and the host cell of ``batch``'s system (host reads, once per system; not
        inside a capture); returns the batch."""
        N = batch.n_real
        elem = batch.species[:N].long() - 1
        if int(elem.min()) < 0 or int(elem.max()) >= self.config.n_elements:
            raise ValueError(f"atomic numbers outside 1..{self.config.n_elements}")
        self._elem = elem.contiguous()
        self._cell_host, self._cell_ptr = _host_cell(batch.cell)
        self._prepared = (batch.species.data_ptr(), batch.cell.data_ptr())
        return batch

    def cell_ptr(self, batch):
        return self._cell_ptr

    def _linear(self, x, weight):
        return wide_gemm.linear(x, weight, precision=self.precision)

    def energy_forces(self, batch, n_systems: int = 1) -> tuple[Tensor, Tensor]:
        """(energy [1] fp64, forces [N, 3]) of one system; capturable in a CUDA graph once ``prepare``
        ran for the system (no host synchronisation)."""
        if n_systems != 1:
            raise ValueError("the NequIP model evaluates one system per batch")
        if getattr(self, "_prepared", None) != (batch.species.data_ptr(), batch.cell.data_ptr()):
            self.prepare(batch)
        c = self.config
        N = batch.n_real
        elem = self._elem
        with torch.enable_grad():
            pos = batch.positions.detach().requires_grad_(True)
            Y, B = _EdgeBasis.apply(pos, self, batch)
            # node features as planes [N (2l + 1), mult]; l = 1, 2 start at exact zeros
            x = [self.w["embed"][elem], None, None]
            # the radial networks' first layers of every block in one GEMM (column views, no copies)
            r1 = torch.split(torch.nn.functional.silu(self._linear(B, self.rad1_all)), c.radial_hidden, dim=1)
            for L in range(c.num_layers):
                zero = lambda l: torch.zeros(N * DIM[l], MULT[l], device=self.device)  # noqa: E731
                # a linear map of an exact zero plane is an exact zero plane: not launched
                h = [self._linear(x[l], self.lin[f"L{L}.lin1_{l}"]) if x[l] is not None else zero(l) for l in range(3)]
                sc = _SelfConnection.apply(*[x[l] if x[l] is not None else zero(l) for l in range(3)], elem,
                                           *[self.w[f"L{L}.sc{l}"] for l in range(3)],
                                           *[self.sc_t[f"L{L}.sc{l}"] for l in range(3)])
                r = torch.nn.functional.silu(self._linear(r1[L], self.w[f"L{L}.rad2"]))
                W = self._linear(r, self.w[f"L{L}.rad3"])
                m = _Conv.apply(torch.cat([p.reshape(-1) for p in h]), Y, W.contiguous(), self, batch)
                o = [self._linear(m[l], self.lin[f"L{L}.lin2_{l}"]) for l in range(3)]
                x = list(_Gate.apply(*o, *sc))
            hid = self._linear(x[0].contiguous(), self.w["readout1"])
            e_atom = self._linear(hid, self.w["readout2"])[:, 0] * c.scale + c.shift
            energy = e_atom.double().sum()
            (grad,) = torch.autograd.grad(energy, pos)
        return energy.detach().reshape(1), (-grad[:N]).detach()

    energy_forces_fused = energy_forces


__all__ = ["NequIPConfig", "NequIPModel", "coupling_table", "gate", "init_weights", "PATHS"]
