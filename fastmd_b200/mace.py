"""MACE-architecture potential on the hot-path kernels (configs with ``MACEAdapter``, fastmd/models/mace.py:254).

The reference evaluates MACE through upstream mace-torch 0.3.16
(``ScaleShiftMACE``, mace.py:356-388), which is not part of the reference
tree. This module implements the published MACE architecture (Batatia et al.,
NeurIPS 2022) at the benchmark's hyperparameters -- C channels, hidden irreps
C x 0e + C x 1o, spherical harmonics l <= 1, correlation order 3, 2
interactions, 8 Bessel radial functions with a polynomial cutoff (p = 5),
radial MLP [64, 64, 64], element one-hot over 89 elements -- directly on
libfastmd_b200 kernels:

* edge geometry and radial basis: ``fmd_mace_edge_geometry`` (one kernel for
  all layers);
* radial MLP and every channel mixing: ``fmd_gemm_f32`` (IEEE FP32; the SiLU
  backward fused into the next GEMM's operand load);
* gather -> tensor-product message -> receiver segment sum:
  ``fmd_mace_message`` (one CTA per receiver, no atomics);
* symmetric contraction: ``fmd_mace_product``; element skip connection:
  ``fmd_element_linear``; energies: ``fmd_mace_node_energy``.

The backward (forces = -dE/dr) is written out kernel by kernel
(``energy_forces``) and also exposed through ``torch.autograd`` (``node_energy``)
so the engine-owned ``EnergyDerivative`` drives it like any energy tap. All
buffers are allocated once per (atoms, edge capacity): a step allocates
nothing and is CUDA-graph capturable.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch
from torch import Tensor

from fastmd_b200 import _lib
from fastmd_b200._lib import call, ptr, stream

ELEMENTS = 89  # one-hot over Z = 1..89 (the benchmark's "89 element embeddings")
RADIAL_PRECISIONS = ("auto", "tf32x3", "ieee")
# the captured-mode row threshold of the reference's 3xTF32 wide GEMMs (fastmd/config.py:153)
# the whole-step crossover measured on a B200 (us per MD step, SIMT edge kernels / tensor-core radial path):
# 1 replica (2.2k edge rows) 151 / 305, 2 replicas 216 / 312, 4 replicas (8.8k rows) 370 / 355,
# 8 replicas 604 / 418, 32 replicas 2160 / 810
RADIAL_TC_MIN_EDGES = 8192


@dataclass(frozen=True)
class MACEConfig:
    channels: int = 128
    num_interactions: int = 2
    correlation: int = 3
    l_max: int = 1
    num_bessel: int = 8
    r_max: float = 6.0
    poly_p: int = 5
    radial_hidden: tuple = (64, 64, 64)
    num_elements: int = ELEMENTS
    readout_hidden: int = 16
    avg_num_neighbors: float = 15.0
    scale: float = 40.0
    shift: float = 0.0

    def paths(self, layer: int) -> int:
        """Tensor-product paths of a layer: 0x0->0, 0x1->1 (+ 1x0->1, 1x1->0 with vector input)."""
        return 2 if layer == 0 else 4


def init_weights(config: MACEConfig, seed: int = 1) -> dict[str, np.ndarray]:
    """Random weights of the architecture (float32, fan-in scaled normals; E0 float64), from
    ``torch.Generator().manual_seed(seed)`` on the CPU: the same bits on every machine."""
    g = torch.Generator().manual_seed(int(seed))
    C, Z = config.channels, config.num_elements

    def normal(*shape, fan_in=None, scale=1.0):
        fan = shape[-1] if fan_in is None else fan_in
        return (torch.randn(*shape, generator=g, dtype=torch.float32) * (scale / math.sqrt(fan))).numpy()

    gain = 1.679  # second-moment gain of SiLU: keeps the radial MLP's activations O(1)

    w: dict[str, np.ndarray] = {"embedding": normal(Z, C, fan_in=1, scale=1.0)}
    for t in range(config.num_interactions):
        last = t == config.num_interactions - 1
        P = config.paths(t)
        h = config.radial_hidden
        w[f"{t}.radial.0"] = normal(h[0], config.num_bessel, scale=gain)
        w[f"{t}.radial.1"] = normal(h[1], h[0], scale=gain)
        w[f"{t}.radial.2"] = normal(h[2], h[1], scale=gain)
        w[f"{t}.radial.3"] = normal(P * C, h[2], scale=gain)
        w[f"{t}.up0"] = normal(C, C)
        if t > 0:
            w[f"{t}.up1"] = normal(C, C)
        w[f"{t}.lin0"] = normal(C, C)
        w[f"{t}.lin1"] = normal(C, C)
        w[f"{t}.prod0"] = normal(Z, 5, C, fan_in=1, scale=0.3)
        if not last:
            w[f"{t}.prod1"] = normal(Z, 4, C, fan_in=1, scale=0.3)
            w[f"{t}.out1"] = normal(C, C)
        w[f"{t}.out0"] = normal(C, C)
        if t > 0:
            w[f"{t}.skip0"] = normal(Z, C, C, fan_in=C)
            if not last:
                w[f"{t}.skip1"] = normal(Z, C, C, fan_in=C)
    w["readout.0"] = normal(1, C)
    w["readout.1a"] = normal(config.readout_hidden, C)
    w["readout.1b"] = normal(1, config.readout_hidden)
    w["e0"] = (torch.randn(Z, generator=g, dtype=torch.float64) * 2.0 - 3.0).numpy()
    return w


def element_index(atomic_numbers) -> np.ndarray:
    z = np.asarray(atomic_numbers, dtype=np.int64)
    if np.any((z < 1) | (z > ELEMENTS)):
        raise ValueError(f"the model covers atomic numbers 1..{ELEMENTS}")
    return (z - 1).astype(np.int32)


def _gemm(a, w, y, *, trans_w=True, a_pre=None, bias=None, y_pre=None, act=0, accumulate=False, m=None,
          n=None, k=None, s=None):
    """y = act(a' . op(w) + bias) on rows of contiguous row-major matrices."""
    m = a.shape[0] if m is None else m
    k = (w.shape[1] if trans_w else w.shape[0]) if k is None else k
    n = (w.shape[0] if trans_w else w.shape[1]) if n is None else n
    call("fmd_gemm_f32", ptr(a), a.stride(0), ptr(a_pre), a_pre.stride(0) if a_pre is not None else 0, ptr(w),
         w.stride(0), int(trans_w), ptr(bias), ptr(y), y.stride(0), ptr(y_pre),
         y_pre.stride(0) if y_pre is not None else 0, m, n, k, act, int(accumulate), s)


@dataclass
class _Buffers:
    """Persistent activations of one (atoms, edges) size."""

    n_atoms: int
    n_edges: int
    t: dict = field(default_factory=dict)


class MACEModel:
    """The potential on one device: ``energy_forces(batch)`` (explicit backward) and
    ``node_energy(inputs, positions, cell)`` (autograd energy tap)."""

    name = "mace"

    def __init__(self, config: MACEConfig | None = None, weights: dict | None = None, *, seed: int = 1,
                 device="cuda", radial_precision: str = "auto") -> None:
        self.config = config or MACEConfig()
        if radial_precision not in RADIAL_PRECISIONS:
            raise ValueError(f"radial_precision must be one of {RADIAL_PRECISIONS}")
        # the fused step's radial MLPs: tcgen05 3xTF32 GEMMs from this many edge rows on, else the
        # IEEE FP32 edge kernels ("auto": from the measured crossover of the two paths, 8,192 rows)
        self.radial_tc_min_edges = {"auto": RADIAL_TC_MIN_EDGES, "tf32x3": 1, "ieee": 0}[radial_precision]
        if self.config.l_max != 1 or self.config.correlation != 3:
            raise ValueError("this build implements l_max = 1 and correlation = 3")
        if self.config.channels % 32 != 0:
            raise ValueError("channels must be a multiple of 32")
        self.device = torch.device(device)
        _lib.require_cuda(torch.empty(0, device=self.device))
        host = init_weights(self.config, seed) if weights is None else weights
        self.weights_host = host
        self.w = {k: torch.from_numpy(np.ascontiguousarray(v)).to(self.device) for k, v in host.items()}
        self._buffers: dict[tuple, _Buffers] = {}

    # ------------------------------------------------------------------ buffers
    def buffers(self, n_atoms: int, n_edges: int) -> _Buffers:
        key = (n_atoms, n_edges)
        buf = self._buffers.get(key)
        if buf is not None:
            return buf
        c = self.config
        C, N, E = c.channels, n_atoms, n_edges
        dev = self.device

        def z(*shape, dtype=torch.float32):
            return torch.zeros(*shape, dtype=dtype, device=dev)

        t = {"ysh": z(E, 4), "phi": z(E, c.num_bessel), "s0": z(N, C),
             "gY": z(E, 3), "gphi": z(E, c.num_bessel), "e_terms": z(2, N), "node_energy": z(N, dtype=torch.float64),
             "d_term": z(N), "readout_pre": z(N, c.readout_hidden), "readout_h": z(N, c.readout_hidden),
             "dh_read": z(N, c.readout_hidden), "dpos": z(N, 3)}
        h = c.radial_hidden
        for L in range(c.num_interactions):
            P = c.paths(L)
            for name, shape in (("pre1", (E, h[0])), ("h1", (E, h[0])), ("pre2", (E, h[1])), ("h2", (E, h[1])),
                                ("pre3", (E, h[2])), ("h3", (E, h[2])), ("R", (E, P * C)), ("dR", (E, P * C)),
                                ("dh3", (E, h[2])), ("dh2", (E, h[1])), ("dh1", (E, h[0])),
                                ("s_t", (N, C)), ("v_t", (N, 3, C)), ("A0", (N, C)), ("A1", (N, 3, C)),
                                ("A0l", (N, C)), ("A1l", (N, 3, C)), ("B0", (N, C)), ("B1", (N, 3, C)),
                                ("s", (N, C)), ("v", (N, 3, C)), ("ds", (N, C)), ("dv", (N, 3, C)),
                                ("dB0", (N, C)), ("dB1", (N, 3, C)), ("dA0l", (N, C)), ("dA1l", (N, 3, C)),
                                ("dA0", (N, C)), ("dA1", (N, 3, C)), ("ds_t", (N, C)), ("dv_t", (N, 3, C))):
                t[f"{L}.{name}"] = z(*shape)
        buf = _Buffers(N, E, t)
        self._buffers[key] = buf
        return buf

    # ------------------------------------------------------------------ forward
    def forward(self, batch, positions: Tensor | None = None, cell: Tensor | None = None,
                buf: _Buffers | None = None) -> _Buffers:
        """Node energies of ``batch`` (a graph batch of fmd_refilter_edges); leaves every
        activation the backward needs in the buffers."""
        c = self.config
        C = c.channels
        pos = batch.positions if positions is None else positions
        cell = batch.cell if cell is None else cell
        N = pos.shape[0]
        E = batch.edge_index.shape[0]
        buf = self.buffers(N, E) if buf is None else buf
        b, w = buf.t, self.w
        s = stream(self.device)
        elem = batch.element
        call("fmd_mace_edge_geometry", ptr(pos), ptr(cell), ptr(batch.edge_index), ptr(batch.edge_image), E,
             c.r_max, c.num_bessel, c.poly_p, ptr(b["ysh"]), ptr(b["phi"]), s)
        # embedding: one-hot(z) @ W is the element's row, one gather
        parts = (_lib.FmdCatPart * 1)()
        parts[0].src, parts[0].index, parts[0].ld = ptr(w["embedding"]), ptr(batch.element64), C
        parts[0].n_src, parts[0].width = c.num_elements, C
        call("fmd_gather_cat", parts, 1, N, ptr(b["s0"]), C, ptr(_lib.flags_word(self.device)), s)
        s_in, v_in = b["s0"], None
        inv_avg = 1.0 / c.avg_num_neighbors
        for L in range(c.num_interactions):
            last = L == c.num_interactions - 1
            P = c.paths(L)
            p = f"{L}."
            # radial MLP phi -> R
            _gemm(b["phi"], w[p + "radial.0"], b[p + "h1"], y_pre=b[p + "pre1"], act=1, s=s)
            _gemm(b[p + "h1"], w[p + "radial.1"], b[p + "h2"], y_pre=b[p + "pre2"], act=1, s=s)
            _gemm(b[p + "h2"], w[p + "radial.2"], b[p + "h3"], y_pre=b[p + "pre3"], act=1, s=s)
            _gemm(b[p + "h3"], w[p + "radial.3"], b[p + "R"], s=s)
            # linear up
            _gemm(s_in, w[p + "up0"], b[p + "s_t"], s=s)
            if v_in is not None:
                _gemm(v_in.view(3 * N, C), w[p + "up1"], b[p + "v_t"].view(3 * N, C), s=s)
            call("fmd_mace_message", ptr(b[p + "R"]), P, ptr(b[p + "s_t"]),
                 ptr(b[p + "v_t"]) if P == 4 else None, ptr(b["ysh"]), ptr(batch.edge_index), ptr(batch.recv_off),
                 N, C, inv_avg, ptr(b[p + "A0"]), ptr(b[p + "A1"]), s)
            _gemm(b[p + "A0"], w[p + "lin0"], b[p + "A0l"], s=s)
            _gemm(b[p + "A1"].view(3 * N, C), w[p + "lin1"], b[p + "A1l"].view(3 * N, C), s=s)
            call("fmd_mace_product", ptr(b[p + "A0l"]), ptr(b[p + "A1l"]), ptr(elem), ptr(w[p + "prod0"]),
                 ptr(w.get(p + "prod1")) if not last else None, N, C, ptr(b[p + "B0"]),
                 ptr(b[p + "B1"]) if not last else None, s)
            _gemm(b[p + "B0"], w[p + "out0"], b[p + "s"], s=s)
            if L > 0:
                call("fmd_element_linear", ptr(s_in), N, 1, ptr(elem), ptr(w[p + "skip0"]), C, C, 0, ptr(b[p + "s"]),
                     1, s)
            if not last:
                _gemm(b[p + "B1"].view(3 * N, C), w[p + "out1"], b[p + "v"].view(3 * N, C), s=s)
                if L > 0 and v_in is not None:
                    call("fmd_element_linear", ptr(v_in), 3 * N, 3, ptr(elem), ptr(w[p + "skip1"]), C, C, 0,
                         ptr(b[p + "v"]), 1, s)
            # readouts
            if L == 0:
                _gemm(b[p + "s"], w["readout.0"], b["e_terms"][0].view(N, 1), s=s)
            if last:
                _gemm(b[p + "s"], w["readout.1a"], b["readout_h"], y_pre=b["readout_pre"], act=1, s=s)
                _gemm(b["readout_h"], w["readout.1b"], b["e_terms"][1].view(N, 1), s=s)
            s_in, v_in = b[p + "s"], (b[p + "v"] if not last else None)
        return buf

    def energies(self, batch, buf: _Buffers, n_systems: int) -> Tensor:
        """Per-system fp64 total energies (and buf['node_energy'])."""
        N = buf.n_atoms
        key = f"total{n_systems}"
        if key not in buf.t:
            buf.t[key] = torch.zeros(n_systems, dtype=torch.float64, device=self.device)
        total = buf.t[key]
        elem = batch.element
        call("fmd_mace_node_energy", ptr(buf.t["e_terms"]), 2, N, ptr(elem), ptr(self.w["e0"]), self.config.scale,
             self.config.shift, N // n_systems, n_systems, ptr(buf.t["node_energy"]), ptr(total), stream(self.device))
        return total

    # ----------------------------------------------------------------- backward
    def backward(self, batch, buf: _Buffers, d_term: Tensor, out: Tensor | None = None,
                 sign: float = 1.0) -> Tensor:
        """``sign * dE/dpositions`` [N, 3] (into ``out``, default buf['dpos']) given the gradient of
        every node's energy terms (``d_term`` [N], i.e. scale * dE/dE_i)."""
        c = self.config
        C = c.channels
        b, w = buf.t, self.w
        N = buf.n_atoms
        s = stream(self.device)
        elem = batch.element
        inv_avg = 1.0 / c.avg_num_neighbors
        Lmax = c.num_interactions - 1
        # last readout: e1 = rb . silu(ra s)
        _gemm(d_term.view(N, 1), w["readout.1b"], b["dh_read"], trans_w=False, s=s)
        _gemm(b["dh_read"], w["readout.1a"], b[f"{Lmax}.ds"], trans_w=False, a_pre=b["readout_pre"], s=s)
        have_dv = False
        for L in range(Lmax, -1, -1):
            last = L == Lmax
            P = c.paths(L)
            p = f"{L}."
            if L == 0:  # first readout: e0 = r0 . s
                # layer 0's output also feeds the linear readout (ds already holds its other uses)
                _gemm(d_term.view(N, 1), w["readout.0"], b[p + "ds"], trans_w=False, accumulate=True, s=s)
            # out-linears
            _gemm(b[p + "ds"], w[p + "out0"], b[p + "dB0"], trans_w=False, s=s)
            if not last:
                _gemm(b[p + "dv"].view(3 * N, C), w[p + "out1"], b[p + "dB1"].view(3 * N, C), trans_w=False, s=s)
            call("fmd_mace_product_bwd", ptr(b[p + "dB0"]), ptr(b[p + "dB1"]) if not last else None,
                 ptr(b[p + "A0l"]), ptr(b[p + "A1l"]), ptr(elem), ptr(w[p + "prod0"]),
                 ptr(w.get(p + "prod1")) if not last else None, N, C, ptr(b[p + "dA0l"]), ptr(b[p + "dA1l"]), s)
            _gemm(b[p + "dA0l"], w[p + "lin0"], b[p + "dA0"], trans_w=False, s=s)
            _gemm(b[p + "dA1l"].view(3 * N, C), w[p + "lin1"], b[p + "dA1"].view(3 * N, C), trans_w=False, s=s)
            call("fmd_mace_message_bwd", ptr(b[p + "dA0"]), ptr(b[p + "dA1"]), ptr(b[p + "R"]), P,
                 ptr(b[p + "s_t"]), ptr(b[p + "v_t"]) if P == 4 else None, ptr(b["ysh"]), ptr(batch.edge_index),
                 ptr(batch.recv_off), ptr(batch.send_off), ptr(batch.send_perm), N, C, inv_avg, ptr(b[p + "dR"]),
                 ptr(b["gY"]), int(L != Lmax), ptr(b[p + "ds_t"]), ptr(b[p + "dv_t"]) if P == 4 else None, s)
            # radial MLP backward into gphi (the layers accumulate)
            _gemm(b[p + "dR"], w[p + "radial.3"], b[p + "dh3"], trans_w=False, s=s)
            _gemm(b[p + "dh3"], w[p + "radial.2"], b[p + "dh2"], trans_w=False, a_pre=b[p + "pre3"], s=s)
            _gemm(b[p + "dh2"], w[p + "radial.1"], b[p + "dh1"], trans_w=False, a_pre=b[p + "pre2"], s=s)
            _gemm(b[p + "dh1"], w[p + "radial.0"], b["gphi"], trans_w=False, a_pre=b[p + "pre1"],
                  accumulate=L != Lmax, s=s)
            if L == 0:
                break
            q = f"{L - 1}."
            # into the previous layer's outputs: linear up and the skip connection
            _gemm(b[p + "ds_t"], w[p + "up0"], b[q + "ds"], trans_w=False, s=s)
            call("fmd_element_linear", ptr(b[p + "ds"]), N, 1, ptr(elem), ptr(w[p + "skip0"]), C, C, 1,
                 ptr(b[q + "ds"]), 1, s)
            _gemm(b[p + "dv_t"].view(3 * N, C), w[p + "up1"], b[q + "dv"].view(3 * N, C), trans_w=False, s=s)
            if not last:
                call("fmd_element_linear", ptr(b[p + "dv"]), 3 * N, 3, ptr(elem), ptr(w[p + "skip1"]), C, C, 1,
                     ptr(b[q + "dv"]), 1, s)
            have_dv = True
        del have_dv
        out = b["dpos"] if out is None else out
        call("fmd_mace_edge_geometry_bwd", ptr(b["ysh"]), ptr(b["gY"]), ptr(b["gphi"]), c.r_max, c.num_bessel,
             c.poly_p, ptr(batch.edge_index), ptr(batch.recv_off), ptr(batch.send_off), ptr(batch.send_perm), N,
             ptr(out), float(sign), 0, s)
        return out

    def cell_grad(self, batch, buf: _Buffers) -> Tensor:
        """d(loss)/d(cell) [3, 3] = sum_e image_e^T g_e after ``backward`` (its edge gradients)."""
        c = self.config
        b = buf.t
        if "virial_ws" not in b:
            b["virial_ws"] = torch.empty(5328, dtype=torch.float64, device=self.device)  # FMD_EDGE_VIRIAL_WORKSPACE_DOUBLES
        out = torch.empty(3, 3, dtype=torch.float32, device=self.device)
        n_real = getattr(batch, "n_edges", None)
        call("fmd_mace_edge_virial", ptr(b["ysh"]), ptr(b["gY"]), ptr(b["gphi"]), c.r_max, c.num_bessel, c.poly_p,
             ptr(batch.edge_image), batch.edge_index.shape[0],
             ptr(n_real) if isinstance(n_real, Tensor) and n_real.is_cuda else None, ptr(b["virial_ws"]), 1.0,
             ptr(out), None, 0, stream(self.device))
        return out

    # ------------------------------------------------------------ entry points
    def prepare(self, batch):
        """Attach the element rows of the batch's atomic numbers (host check, once per system;
        not inside a capture) and return the batch (the adapter's ``prepare``, mace.py:309)."""
        elem = torch.from_numpy(element_index(batch.species.cpu().numpy())).to(self.device)
        batch.element = elem
        batch.element64 = elem.to(torch.int64)
        return batch

    def energy_forces(self, batch, n_systems: int = 1) -> tuple[Tensor, Tensor]:
        """(per-system fp64 energies [R], forces [N, 3] float32) of ``batch``: forward, then the
        explicit backward of the summed energy (forces = -dE/dr). No allocation after the first call."""
        N = batch.positions.shape[0]
        buf = self.buffers(N, batch.edge_index.shape[0])
        if getattr(batch, "element", None) is None:
            self.prepare(batch)
        self.forward(batch, buf=buf)
        total = self.energies(batch, buf, n_systems)
        key = f"ones{n_systems}"
        if key not in buf.t:
            buf.t[key] = torch.ones(n_systems, dtype=torch.float64, device=self.device)
            buf.t["forces"] = torch.zeros(N, 3, dtype=torch.float32, device=self.device)
        call("fmd_mace_node_energy_bwd", ptr(buf.t[key]), self.config.scale, N // n_systems, n_systems,
             ptr(buf.t["d_term"]), stream(self.device))
        forces = self.backward(batch, buf, buf.t["d_term"], out=buf.t["forces"], sign=-1.0)
        return total, forces

    def node_energy(self, inputs, positions: Tensor, cell: Tensor) -> Tensor:
        """Energy tap: per-atom fp64 energies, differentiable with respect to ``positions`` and ``cell``."""
        return _NodeEnergy.apply(positions, cell, self, inputs)


class _NodeEnergy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, positions, cell, model: MACEModel, batch):
        pos = positions.detach().float().contiguous()
        buf = model.buffers(pos.shape[0], batch.edge_index.shape[0])
        if getattr(batch, "element", None) is None:
            model.prepare(batch)
        model.forward(batch, positions=pos, cell=cell.detach().float().contiguous(), buf=buf)
        model.energies(batch, buf, 1)
        ctx.model, ctx.batch, ctx.buf = model, batch, buf
        ctx.pos_dtype, ctx.cell_dtype = positions.dtype, cell.dtype
        return buf.t["node_energy"].clone()

    @staticmethod
    def backward(ctx, grad_node):
        model, buf = ctx.model, ctx.buf
        d_term = buf.t["d_term"]
        torch.mul(grad_node.to(torch.float32), float(model.config.scale), out=d_term)
        dpos = torch.empty(buf.n_atoms, 3, dtype=torch.float32, device=d_term.device)
        model.backward(ctx.batch, buf, d_term, out=dpos)
        dcell = None
        if ctx.needs_input_grad[1]:  # the strain leaf of a stress: d(loss)/d(cell) over the edge images
            dcell = model.cell_grad(ctx.batch, buf).to(ctx.cell_dtype)
        return dpos.to(ctx.pos_dtype), dcell, None, None


# --------------------------------------------------------------------------- fused step

_L = 4  # FMD_MACE_MAX_LAYERS
_FP = ctypes_fp = None


def _struct_types():
    import ctypes

    P = ctypes.c_void_p
    arr = P * _L

    class FusedWeights(ctypes.Structure):
        _fields_ = [(name, arr) for name in (
            "radial_w1t", "radial_w2t", "radial_w3t", "radial_w4t", "radial_w1", "radial_w2", "radial_w3",
            "radial_w4", "lin0", "lin1", "lin0t", "lin1t", "out0", "out1", "out0t", "out1t", "up0", "up1", "up0t",
            "up1t", "prod0", "prod1", "skip0", "skip1", "skip0t", "skip1t")] + [
            ("s_t0", P), ("r0", P), ("ra", P), ("rb", P), ("e0", P), ("scale", ctypes.c_double),
            ("shift", ctypes.c_double), ("n_layers", ctypes.c_int32), ("n_basis", ctypes.c_int32),
            ("poly_p", ctypes.c_int32), ("readout_hidden", ctypes.c_int32), ("radial_hidden", ctypes.c_int32),
            ("r_max", ctypes.c_float), ("inv_avg", ctypes.c_float), ("_pad", ctypes.c_int32)] + [
            (name, arr * 3) for name in ("radial_tc_hi", "radial_tc_lo", "radial_tc_t_hi", "radial_tc_t_lo")] + [
            ("radial_tc_min_edges", ctypes.c_int64), ("node_tc_hi", arr * 12), ("node_tc_lo", arr * 12),
            ("skip_tc_hi", arr * 2), ("skip_tc_lo", arr * 2)]

    class FusedState(ctypes.Structure):
        _fields_ = [(name, arr) for name in (
            "R", "dR", "s_t", "v_t", "A0", "A1", "A0l", "A1l", "s_out", "v_out", "dA0", "dA1", "ds_skip",
            "dv_skip")] + [
            ("ysh", P), ("dY", P), ("g_r", P), ("e_term0", P), ("node_energy", P), ("elem", P), ("groups", P),
            ("n_groups", ctypes.c_int64), ("radial_pre", arr * 3), ("flags", P), ("elem_order", P),
            ("elem_rank", P), ("n_elem_runs", ctypes.c_int64), ("elem_runs_host", P)]

    return FusedWeights, FusedState


_FusedWeights, _FusedState = _struct_types()
_lib.declare("fmd_mace_fused_step", [_lib.ctypes.POINTER(_FusedWeights), _lib.ctypes.POINTER(_FusedState),
                                     *([_lib.c_void_p] * 4), _lib.c_int64, *([_lib.c_void_p] * 4), _lib.c_int64,
                                     _lib.c_int32, _lib.c_int32, _lib.c_void_p, _lib.c_void_p, _lib.c_int32,
                                     _lib.c_void_p])


def _fused_weights(model: "MACEModel"):
    """Device copies of the weights in the layouts the fused kernels read (built once)."""
    c, w, dev = model.config, model.w, model.device
    keep: dict[str, Tensor] = {}

    def t(x):
        return x.t().contiguous()

    fw = _FusedWeights()
    for L in range(c.num_interactions):
        p = f"{L}."
        for k in range(4):
            keep[f"{p}w{k + 1}t"] = t(w[f"{p}radial.{k}"])
            keep[f"{p}w{k + 1}"] = w[f"{p}radial.{k}"].contiguous()
        for name in ("lin0", "lin1", "out0", "out1", "up0", "up1"):
            if p + name in w:
                keep[p + name] = w[p + name].contiguous()
                keep[p + name + "t"] = t(w[p + name])
        for name in ("skip0", "skip1"):
            if p + name in w:
                keep[p + name] = w[p + name].contiguous()
                keep[p + name + "t"] = w[p + name].transpose(1, 2).contiguous()
        for name in ("prod0", "prod1"):
            if p + name in w:
                keep[p + name] = w[p + name].contiguous()
    # layer 0's up-mixing of the embedding, per element, with the GEMM of the unfused path
    table = torch.empty(c.num_elements, c.channels, dtype=torch.float32, device=dev)
    _gemm(w["embedding"], w["0.up0"], table, s=stream(dev))
    keep["s_t0"] = table
    keep["r0"] = w["readout.0"].reshape(-1).contiguous()
    keep["ra"] = w["readout.1a"].contiguous()
    keep["rb"] = w["readout.1b"].reshape(-1).contiguous()
    keep["e0"] = w["e0"].contiguous()

    def q(name):
        return ptr(keep[name]) if name in keep else None

    for L in range(c.num_interactions):
        p = f"{L}."
        for k in range(4):
            getattr(fw, f"radial_w{k + 1}t")[L] = q(f"{p}w{k + 1}t")
            getattr(fw, f"radial_w{k + 1}")[L] = q(f"{p}w{k + 1}")
        for name in ("lin0", "lin1", "out0", "out1", "up0", "up1", "skip0", "skip1"):
            getattr(fw, name)[L] = q(p + name)
            getattr(fw, name + "t")[L] = q(p + name + "t")
        fw.prod0[L] = q(p + "prod0")
        fw.prod1[L] = q(p + "prod1")
    fw.s_t0, fw.r0, fw.ra, fw.rb, fw.e0 = q("s_t0"), q("r0"), q("ra"), q("rb"), q("e0")
    fw.scale, fw.shift = float(c.scale), float(c.shift)
    fw.n_layers, fw.n_basis, fw.poly_p = c.num_interactions, c.num_bessel, c.poly_p
    fw.readout_hidden, fw.radial_hidden = c.readout_hidden, c.radial_hidden[0]
    fw.r_max, fw.inv_avg = float(c.r_max), float(1.0 / c.avg_num_neighbors)
    if len(set(c.radial_hidden)) != 1 or c.radial_hidden[0] != 64:
        raise ValueError("the fused step implements radial MLP widths (64, 64, 64)")
    fw.radial_tc_min_edges = int(model.radial_tc_min_edges)
    if model.radial_tc_min_edges > 0:
        # TF32 hi/lo pairs of W2..W4 as [out][in] (forward) and [in][out] (backward), K-major for TMA
        s = stream(dev)
        for L in range(c.num_interactions):
            for k in range(3):
                wk = w[f"{L}.radial.{k + 1}"].contiguous()
                for transposed, hi_name, lo_name in ((0, "radial_tc_hi", "radial_tc_lo"),
                                                     (1, "radial_tc_t_hi", "radial_tc_t_lo")):
                    rows, cols = wk.shape
                    shape = (cols, rows) if transposed else (rows, cols)
                    hi = torch.empty(shape, dtype=torch.float32, device=dev)
                    lo = torch.empty(shape, dtype=torch.float32, device=dev)
                    call("fmd_tf32_split", ptr(wk), rows, cols, cols, transposed, ptr(hi), ptr(lo), shape[1], s)
                    keep[f"{L}.{hi_name}{k}"], keep[f"{L}.{lo_name}{k}"] = hi, lo
                    getattr(fw, hi_name)[k][L] = ptr(hi)
                    getattr(fw, lo_name)[k][L] = ptr(lo)
        # the node kernels' channel mixings on the tensor cores (a 2-layer model): [out][in] splits for the
        # forward mixings (index m) and [in][out] splits for their backward (6 + m)
        if c.num_interactions == 2:
            for L in range(c.num_interactions):
                for m, name in enumerate(("lin0", "lin1", "out0", "out1", "up0", "up1")):
                    key = f"{L}.{name}"
                    if key not in w or (L == 0 and name in ("up0", "up1")):
                        continue  # layer 0's up-mixing is the embedding table
                    wk = w[key].contiguous()
                    for transposed in (0, 1):
                        hi = torch.empty_like(wk)
                        lo = torch.empty_like(wk)
                        call("fmd_tf32_split", ptr(wk), wk.shape[0], wk.shape[1], wk.shape[1], transposed, ptr(hi),
                             ptr(lo), wk.shape[1], s)
                        idx = m + 6 * transposed
                        keep[f"{key}.ntc_hi{transposed}"], keep[f"{key}.ntc_lo{transposed}"] = hi, lo
                        fw.node_tc_hi[idx][L] = ptr(hi)
                        fw.node_tc_lo[idx][L] = ptr(lo)
                # the per-element skip mixings: skip0t [Z][out][in] (forward) and skip0 [Z][in][out] (backward)
                if f"{L}.skip0" in w:
                    for d, src in enumerate((w[f"{L}.skip0"].transpose(1, 2).contiguous(), w[f"{L}.skip0"].contiguous())):
                        flat = src.reshape(-1, src.shape[-1])
                        hi, lo = torch.empty_like(flat), torch.empty_like(flat)
                        call("fmd_tf32_split", ptr(flat), flat.shape[0], flat.shape[1], flat.shape[1], 0, ptr(hi),
                             ptr(lo), flat.shape[1], s)
                        keep[f"{L}.skip_tc_hi{d}"], keep[f"{L}.skip_tc_lo{d}"] = hi, lo
                        fw.skip_tc_hi[d][L] = ptr(hi)
                        fw.skip_tc_lo[d][L] = ptr(lo)
    return fw, keep


def element_groups(elements: np.ndarray, size: int = 4) -> np.ndarray:
    """Atoms grouped by element, ``size`` per group (-1 padding): the node kernels' work units."""
    groups = []
    for z in np.unique(elements):
        atoms = np.nonzero(elements == z)[0]
        for start in range(0, atoms.size, size):
            chunk = atoms[start:start + size]
            groups.append(np.concatenate([chunk, np.full(size - chunk.size, -1)]))
    return np.asarray(groups, dtype=np.int32).reshape(-1, size)


class _FusedBuffers:
    def __init__(self, model: "MACEModel", n_atoms: int, n_edges: int, elem: Tensor):
        c, dev = model.config, model.device
        C, N, E = c.channels, n_atoms, n_edges
        z = lambda *s, dtype=torch.float32: torch.zeros(*s, dtype=dtype, device=dev)  # noqa: E731
        self.t: dict[str, Tensor] = {}
        st = _FusedState()
        last = c.num_interactions - 1
        for L in range(c.num_interactions):
            P = c.paths(L)
            for name, shape in (("R", (E, P * C)), ("dR", (E, P * C)), ("s_t", (N, C)), ("v_t", (N, 3, C)),
                                ("A0", (N, C)), ("A1", (N, 3, C)), ("A0l", (N, C)), ("A1l", (N, 3, C)),
                                ("s_out", (N, C)), ("v_out", (N, 3, C)), ("dA0", (N, C)), ("dA1", (N, 3, C))):
                self.t[f"{L}.{name}"] = z(*shape)
                getattr(st, name)[L] = ptr(self.t[f"{L}.{name}"])
            if L > 0:
                self.t[f"{L}.ds_skip"] = z(N, C)
                st.ds_skip[L] = ptr(self.t[f"{L}.ds_skip"])
                if L < last:
                    self.t[f"{L}.dv_skip"] = z(N, 3, C)
                    st.dv_skip[L] = ptr(self.t[f"{L}.dv_skip"])
        for name, shape, dtype in (("ysh", (E, 4), torch.float32), ("dY", (E, 3), torch.float32),
                                   ("g_r", (E, 3), torch.float32), ("e_term0", (N,), torch.float32),
                                   ("node_energy", (N,), torch.float64), ("forces", (N, 3), torch.float32)):
            self.t[name] = z(*shape, dtype=dtype)
        groups = torch.from_numpy(element_groups(elem.cpu().numpy())).to(dev)
        self.t["groups"] = groups
        self.t["elem"] = elem
        st.ysh, st.dY, st.g_r = ptr(self.t["ysh"]), ptr(self.t["dY"]), ptr(self.t["g_r"])
        st.e_term0, st.node_energy = ptr(self.t["e_term0"]), ptr(self.t["node_energy"])
        st.elem, st.groups, st.n_groups = ptr(elem), ptr(groups), int(groups.shape[0])
        # the atoms by element for the skip mixings on the tensor cores: order, rank and the element runs
        elem_np = elem.cpu().numpy()
        order = np.argsort(elem_np, kind="stable").astype(np.int32)
        rank = np.empty_like(order)
        rank[order] = np.arange(order.size, dtype=np.int32)
        zs, first, counts = np.unique(elem_np[order], return_index=True, return_counts=True)
        self.elem_runs_host = np.ascontiguousarray(np.stack([zs, first, counts], axis=1).astype(np.int64))
        self.t["elem_order"] = torch.from_numpy(order).to(dev)
        self.t["elem_rank"] = torch.from_numpy(rank).to(dev)
        st.elem_order, st.elem_rank = ptr(self.t["elem_order"]), ptr(self.t["elem_rank"])
        st.n_elem_runs = int(self.elem_runs_host.shape[0])
        st.elem_runs_host = self.elem_runs_host.ctypes.data
        if 0 < model.radial_tc_min_edges <= E:  # the radial pre-activations of the tensor-core path
            for L in range(c.num_interactions):
                for k in range(3):
                    self.t[f"{L}.pre{k}"] = z(E, c.radial_hidden[0])
                    st.radial_pre[k][L] = ptr(self.t[f"{L}.pre{k}"])
        st.flags = ptr(_lib.flags_word(dev))
        self.tensor_core_radial = False  # whether the last step took the tensor-core radial path
        self.tensor_core_nodes = False   # and the node mixings on the tensor cores
        self.state = st
        self.energy: dict[int, Tensor] = {}


def _energy_forces_fused(self: "MACEModel", batch, n_systems: int = 1, stages: int = -1):
    """(per-system fp64 energies [R], forces [N, 3] float32) of ``batch`` in the fused kernels
    (``fmd_mace_fused_step``); the same mathematics as ``energy_forces``."""
    if getattr(batch, "element", None) is None:
        self.prepare(batch)
    N, E = batch.positions.shape[0], batch.edge_index.shape[0]
    if getattr(self, "_fused_w", None) is None:
        self._fused_w = _fused_weights(self)
        self._fused_bufs = {}
    # buffers per (atoms, edge rows rounded up to 256): a ragged build whose edge count drifts
    # reuses them (the kernels touch the first E rows only)
    cap = -(-max(E, 1) // 256) * 256
    key = (N, cap, ptr(batch.element))
    buf = self._fused_bufs.get(key)
    if buf is None:
        buf = _FusedBuffers(self, N, cap, batch.element)
        self._fused_bufs[key] = buf
    buf.tensor_core_radial = 0 < self.radial_tc_min_edges <= E
    # the node kernels' channel mixings on the tensor cores as well (2-layer models)
    buf.tensor_core_nodes = buf.tensor_core_radial and self.config.num_interactions == 2
    if n_systems not in buf.energy:
        buf.energy[n_systems] = torch.zeros(n_systems, dtype=torch.float64, device=self.device)
    energy, forces = buf.energy[n_systems], buf.t["forces"]
    fw, _ = self._fused_w
    import ctypes as _ct

    call("fmd_mace_fused_step", _ct.byref(fw), _ct.byref(buf.state), ptr(batch.positions), ptr(batch.cell),
         ptr(batch.edge_index), ptr(batch.edge_image), E, ptr(batch.n_edges), ptr(batch.recv_off), ptr(batch.send_off),
         ptr(batch.send_perm), N // n_systems, n_systems, self.config.channels, ptr(forces), ptr(energy),
         int(stages), stream(self.device))
    return energy, forces


MACEModel.energy_forces_fused = _energy_forces_fused
