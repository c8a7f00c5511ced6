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
the position gradient: autograd over this build's kernels back to the radial basis and the harmonics
(the convolution and its backward, ``fmd_nequip_conv``; the linears on the tcgen05 wide GEMM,
``precision="tf32x3"``, or its IEEE path, ``"ieee"``), then the edge basis backward
(``fmd_nequip_edge_basis_bwd``) and the forces summed over the receiver and sender CSRs
(``fmd_edge_forces``). Element indices are
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


_ACT_INPUT_SILU, _ACT_SILU_GRAD = 16, 2  # fmd_gemm_tf32x3: SiLU on the operand / times silu'(c)


def _zero(t: Tensor) -> Tensor:
    """``t`` set to zeros by a stream-ordered memset (``fmd_zero``; no kernel)."""
    call("fmd_zero", ptr(t), t.numel() * t.element_size(), stream(t.device))
    return t


def _gemm(model, a: Tensor, w: Tensor, transposed: bool = False, out=None, accumulate: bool = False, act: int = 0,
          c=None, a_pre=None, y_pre=None) -> Tensor:
    """``y (+)= a @ B`` with ``B = w^T`` (or ``w`` when ``transposed``) in the model's precision: the tcgen05
    3xTF32 GEMM (``act``/``c`` its fused SiLU modes; ``accumulate`` adds to ``out``) or the IEEE SIMT GEMM
    (``act = 1`` SiLU output with the pre-activation into ``y_pre``; ``a_pre``: the operand times
    silu'(a_pre) as it is loaded)."""
    m, k = a.shape
    n = w.shape[1] if transposed else w.shape[0]
    y = torch.empty((m, n), device=a.device) if out is None else out
    if m == 0:
        return y
    if model.precision == "tf32x3":
        if accumulate:
            c = y
        return wide_gemm._launch(a, w, transposed, "tf32x3", c=c, out=y, act=act)
    call("fmd_gemm_f32", ptr(a), a.stride(0), ptr(a_pre), a_pre.stride(0) if a_pre is not None else 0, ptr(w),
         w.stride(0), int(not transposed), None, ptr(y), y.stride(0), ptr(y_pre),
         y_pre.stride(0) if y_pre is not None else 0, m, n, k, act, int(accumulate), stream(a.device))
    return y


def _gemms(model, specs) -> list[Tensor]:
    """Several independent ``_gemm`` calls: on the tensor cores up to four per launch
    (``fmd_gemm_tf32x3_grouped``, each result bitwise that of its own launch); on the IEEE path one by one.
    A spec is a dict with keys a, w and optionally transposed, out, accumulate, act, c."""
    if model.precision != "tf32x3":
        return [_gemm(model, q["a"], q["w"], q.get("transposed", False), out=q.get("out"),
                      accumulate=q.get("accumulate", False), act=q.get("act", 0), c=q.get("c")) for q in specs]
    outs = []
    for i in range(0, len(specs), 4):
        group = []
        for q in specs[i:i + 4]:
            c = q.get("c")
            if q.get("accumulate", False):
                c = q["out"]
            group.append({"a": q["a"], "weight": q["w"], "transposed": q.get("transposed", False), "c": c,
                          "out": q.get("out"), "act": q.get("act", 0)})
        outs.extend(wide_gemm.grouped(group))
    return outs


def _planes(flat: Tensor, n: int, mults) -> tuple[Tensor, ...]:
    """The l planes of a planar buffer as [n (2l + 1), mult] matrices (views)."""
    out, off = [], 0
    for m, d in zip(mults, DIM):
        out.append(flat[off:off + n * m * d].view(n * d, m))
        off += n * m * d
    return tuple(out)


class _RadialNet(Function):
    """The path weights W_L [E, 960] of every block from the radial basis B [E, n_basis]: the blocks' first
    layers as one GEMM (p1 = B W1^T, their weights stacked), then per block W_L = silu(silu(p1_L) W2^T) W3^T
    with each SiLU applied to the next GEMM's operand; the backward forms every silu' product in a GEMM
    epilogue and writes each block's first-layer gradient into its column block, so dB is one GEMM."""

    @staticmethod
    def forward(ctx, B, model):
        c, H = model.config, model.config.radial_hidden
        E = B.shape[0]
        ws = model.w
        p2s, Ws = [], []
        if model.precision == "tf32x3":
            p1 = _gemm(model, B, model.rad1_all)
            layers = range(c.num_layers)
            p2s = _gemms(model, [{"a": p1[:, L * H:(L + 1) * H], "w": ws[f"L{L}.rad2"], "act": _ACT_INPUT_SILU}
                                 for L in layers])
            Ws = _gemms(model, [{"a": p2s[L], "w": ws[f"L{L}.rad3"], "act": _ACT_INPUT_SILU} for L in layers])
        else:
            p1 = torch.empty((E, c.num_layers * H), device=B.device)
            a1 = _gemm(model, B, model.rad1_all, act=1, y_pre=p1)
            for L in range(c.num_layers):
                p2 = torch.empty((E, H), device=B.device)
                a2 = _gemm(model, a1[:, L * H:(L + 1) * H], ws[f"L{L}.rad2"], act=1, y_pre=p2)
                Ws.append(_gemm(model, a2, ws[f"L{L}.rad3"]))
                p2s.append(p2)
        ctx.save_for_backward(p1, *p2s)
        ctx.model = model
        ctx.set_materialize_grads(False)
        return tuple(Ws)

    @staticmethod
    def backward(ctx, *dWs):
        p1, *p2s = ctx.saved_tensors
        model = ctx.model
        H, ws = model.config.radial_hidden, model.w
        g1 = torch.empty_like(p1)
        if any(d is None for d in dWs):
            _zero(g1)
        live = [L for L, dW in enumerate(dWs) if dW is not None]
        blk = lambda L: slice(L * H, (L + 1) * H)  # noqa: E731
        if model.precision == "tf32x3":
            g2s = _gemms(model, [{"a": dWs[L].contiguous(), "w": ws[f"L{L}.rad3"], "transposed": True,
                                  "act": _ACT_SILU_GRAD, "c": p2s[L]} for L in live])
            _gemms(model, [{"a": g2, "w": ws[f"L{L}.rad2"], "transposed": True, "out": g1[:, blk(L)],
                            "act": _ACT_SILU_GRAD, "c": p1[:, blk(L)]} for L, g2 in zip(live, g2s)])
        else:
            for L in live:
                da2 = _gemm(model, dWs[L].contiguous(), ws[f"L{L}.rad3"], True)
                _gemm(model, da2, ws[f"L{L}.rad2"], True, out=g1[:, blk(L)], a_pre=p2s[L])
        if model.precision == "tf32x3":
            dB = _gemm(model, g1, model.rad1_all, True)
        else:
            dB = _gemm(model, g1, model.rad1_all, True, a_pre=p1)
        return dB, None


class _NodeIn(Function):
    """A block's inputs from the node features (planes x0 [N, 128], x1 [3N, 64], x2 [5N, 32]; x1 and x2
    None in the first block, exact zeros): the first linear of each plane written into one planar buffer
    h (the convolution's input) and the element-dependent self-connection planes sc0, sc1, sc2
    (``fmd_nequip_self_connection``). The backward adds the linears' input gradients to the
    self-connection's (the GEMM accumulating into it)."""

    @staticmethod
    def forward(ctx, x0, x1, x2, model, L):
        N, dev = x0.shape[0], x0.device
        first = x1 is None
        if first:
            zeros = _zero(torch.empty(N * (3 * 64 + 5 * 32), device=dev))
            x1, x2 = zeros[:N * 192].view(3 * N, 64), zeros[N * 192:].view(5 * N, 32)
        h = torch.empty(N * X_WIDTH, device=dev)
        hp = _planes(h, N, MULT)
        xs = (x0.contiguous(), x1.contiguous(), x2.contiguous())
        if first:
            _zero(h[N * MULT[0]:])  # a linear map of an exact zero plane is an exact zero plane
        _gemms(model, [{"a": xs[l], "w": model.lin[f"L{L}.lin1_{l}"], "out": hp[l]} for l in range(1 if first else 3)])
        sc = [torch.empty_like(t) for t in xs]
        call("fmd_nequip_self_connection", ptr(xs[0]), ptr(xs[1]), ptr(xs[2]), ptr(model._elem),
             *[ptr(model.w[f"L{L}.sc{l}"]) for l in range(3)], N, 0, ptr(sc[0]), ptr(sc[1]), ptr(sc[2]),
             stream(dev))
        ctx.model, ctx.L, ctx.first, ctx.n = model, L, first, N
        ctx.set_materialize_grads(False)
        return h, sc[0], sc[1], sc[2]

    @staticmethod
    def backward(ctx, dh, d0, d1, d2):
        model, L, N = ctx.model, ctx.L, ctx.n
        dev = model.device
        gs = [g.contiguous() if g is not None else None for g in (d0, d1, d2)]
        shapes = ((N, 128), (3 * N, 64), (5 * N, 32))
        for l in range(3):
            if gs[l] is None:
                gs[l] = _zero(torch.empty(shapes[l], device=dev))
        dx = [torch.empty_like(g) for g in gs]
        call("fmd_nequip_self_connection", ptr(gs[0]), ptr(gs[1]), ptr(gs[2]), ptr(model._elem),
             *[ptr(model.sc_t[f"L{L}.sc{l}"]) for l in range(3)], N, 0, ptr(dx[0]), ptr(dx[1]), ptr(dx[2]),
             stream(dev))
        if dh is not None:
            dhp = _planes(dh.contiguous(), N, MULT)
            _gemms(model, [{"a": dhp[l], "w": model.lin[f"L{L}.lin1_{l}"], "transposed": True, "out": dx[l],
                            "accumulate": True} for l in range(1 if ctx.first else 3)])
        if ctx.first:
            return dx[0], None, None, None, None
        return dx[0], dx[1], dx[2], None, None


class _Conv(Function):
    """Messages (the planar buffer of 3136 N floats: [N, 224] | [N, 3, 384] | [N, 5, 352]) of the block's
    planar input h; the backward returns the gradients of h and W and adds the harmonics' gradient into
    the model's per-evaluation dY buffer (the last block's backward, which runs first, writes it)."""

    @staticmethod
    def forward(ctx, h, W, model, batch, L):
        N = batch.n_real
        m = torch.empty(N * sum(M_MULT[l] * DIM[l] for l in range(3)), device=h.device)
        call("fmd_nequip_conv", ptr(h), ptr(model._Y), ptr(W), ptr(model.cg), ptr(batch.edge_index),
             ptr(batch.recv_off), N, 1.0 / model.config.avg_num_neighbors, ptr(m), stream(h.device))
        ctx.save_for_backward(h, W)
        ctx.model, ctx.batch, ctx.L = model, batch, L
        ctx.set_materialize_grads(False)
        return m

    @staticmethod
    def backward(ctx, dm):
        h, W = ctx.saved_tensors
        model, batch, L = ctx.model, ctx.batch, ctx.L
        last = L == model.config.num_layers - 1
        if dm is None:
            if last:
                _zero(model._dY)
            return None, None, None, None, None
        N = batch.n_real
        # the first block's input (the embedding and exact-zero planes) needs no gradient: dx not formed
        gx = torch.empty_like(h) if ctx.needs_input_grad[0] else None
        gW = torch.empty_like(W)
        call("fmd_nequip_conv_bwd", ptr(h), ptr(model._Y), ptr(W), ptr(model.cg), ptr(batch.edge_index),
             ptr(batch.recv_off), ptr(batch.send_off), ptr(batch.send_perm), N,
             1.0 / model.config.avg_num_neighbors, ptr(dm.contiguous()), ptr(gx), ptr(gW), ptr(model._dY),
             int(not last), stream(h.device))
        return gx, gW, None, None, None


class _PlanarOut(Function):
    """The second linear of each message plane (o0 [N, 224], o1 [3N, 64], o2 [5N, 32]); the backward
    writes the three input gradients into the planes of one buffer (the convolution's gradient input)."""

    @staticmethod
    def forward(ctx, m, model, L):
        N = model._n
        mp = _planes(m, N, M_MULT)
        ctx.model, ctx.L = model, L
        ctx.set_materialize_grads(False)
        return tuple(_gemms(model, [{"a": mp[l], "w": model.lin[f"L{L}.lin2_{l}"]} for l in range(3)]))

    @staticmethod
    def backward(ctx, d0, d1, d2):
        model, L = ctx.model, ctx.L
        N = model._n
        dm = torch.empty(N * sum(M_MULT[l] * DIM[l] for l in range(3)), device=model.device)
        dmp = _planes(dm, N, M_MULT)
        specs = []
        for l, g in enumerate((d0, d1, d2)):
            if g is None:
                _zero(dmp[l])
            else:
                specs.append({"a": g.contiguous(), "w": model.lin[f"L{L}.lin2_{l}"], "transposed": True, "out": dmp[l]})
        _gemms(model, specs)
        return dm, None, None


class _Readout(Function):
    """The system energy (FP64 [1]): e_i = (x0_i W1^T) W2^T scaled and shifted, summed in FP64
    (``fmd_mace_node_energy``: fixed-order block tree). The readout is linear, so the backward is the
    outer product of dE/de_i (``fmd_mace_node_energy_bwd``) with the row v = W2 W1."""

    @staticmethod
    def forward(ctx, x0, model):
        N, c = x0.shape[0], model.config
        hid = _gemm(model, x0.contiguous(), model.w["readout1"])
        out = _gemm(model, hid, model.w["readout2"])
        node = torch.empty(N, dtype=torch.float64, device=x0.device)
        total = torch.empty(1, dtype=torch.float64, device=x0.device)
        call("fmd_mace_node_energy", ptr(out), 1, N, ptr(model._elem32), ptr(model._e0), float(c.scale),
             float(c.shift), N, 1, ptr(node), ptr(total), stream(x0.device))
        ctx.model, ctx.n = model, N
        return total

    @staticmethod
    def backward(ctx, d_total):
        model, N = ctx.model, ctx.n
        dev = model.device
        d_term = torch.empty((N, 1), device=dev)
        call("fmd_mace_node_energy_bwd", ptr(d_total.contiguous()), float(model.config.scale), N, 1, ptr(d_term),
             stream(dev))
        dx0 = torch.empty((N, MULT[0]), device=dev)
        call("fmd_gemm_f32", ptr(d_term), 1, None, 0, ptr(model._readout_row), 1, 1, None, ptr(dx0), MULT[0], None,
             0, N, MULT[0], 1, 0, 0, stream(dev))
        return dx0, None


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
        ctx.set_materialize_grads(False)  # the last block's x1, x2 feed nothing: zeros by memset below
        return tuple(x)

    @staticmethod
    def backward(ctx, dx0, dx1, dx2):
        o0, o1, o2 = ctx.saved_tensors
        n = o0.shape[0]
        dx = [g.contiguous() if g is not None else _zero(torch.empty(n * DIM[l], MULT[l], device=o0.device))
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
        # the linear readout folded to one row for its backward: d e_i / d x0_i = W2 W1 (FP64 product)
        row = host["readout2"].astype(np.float64) @ host["readout1"].astype(np.float64)
        self._readout_row = torch.as_tensor(row.reshape(-1, 1), dtype=torch.float32, device=self.device)
        self._e0 = torch.zeros(self.config.n_elements, dtype=torch.float64, device=self.device)
        self._one = torch.ones(1, dtype=torch.float64, device=self.device)  # dE/dE, made once

    # ------------------------------------------------------------ per-system state (no host work per call)
    def prepare(self, batch):
        """The element rows and the host cell of ``batch``'s system (host reads, once per system; not
        inside a capture); returns the batch."""
        N = batch.n_real
        elem = batch.species[:N].long() - 1
        if int(elem.min()) < 0 or int(elem.max()) >= self.config.n_elements:
            raise ValueError(f"atomic numbers outside 1..{self.config.n_elements}")
        self._elem = elem.contiguous()
        self._elem32 = elem.to(torch.int32).contiguous()
        self._cell_host, self._cell_ptr = _host_cell(batch.cell)
        self._prepared = (batch.species.data_ptr(), batch.cell.data_ptr())
        return batch

    def cell_ptr(self, batch):
        return self._cell_ptr

    def energy_forces(self, batch, n_systems: int = 1) -> tuple[Tensor, Tensor]:
        """(energy [1] fp64, forces [N, 3]) of one system; capturable in a CUDA graph once ``prepare``
        ran for the system (no host synchronisation). Every launch is one of this library's kernels (or a
        memset): the edge basis, the radial network, per block the node inputs, the convolution, the
        second linears and the gate, the FP64 readout; autograd back to the radial basis (the
        convolutions add the harmonics' gradient into one buffer), the basis backward, and the forces
        summed over the receiver and sender CSRs (``fmd_edge_forces``)."""
        if n_systems != 1:
            raise ValueError("the NequIP model evaluates one system per batch")
        if getattr(self, "_prepared", None) != (batch.species.data_ptr(), batch.cell.data_ptr()):
            self.prepare(batch)
        c = self.config
        N = batch.n_real
        dev = self.device
        E = int(batch.edge_index.shape[0])
        self._n = N
        Y = torch.empty(E, 9, device=dev)
        B = torch.empty(E, c.num_bessel, device=dev)
        geo = torch.empty(E, 4, device=dev)
        override = getattr(batch, "edge_vec_override", None)
        n_real_edges = ptr(batch.n_edges) if override is not None else None
        call("fmd_nequip_edge_basis", ptr(batch.positions), self._cell_ptr, ptr(batch.edge_index),
             ptr(batch.edge_image), ptr(override), n_real_edges, E, c.r_max, c.num_bessel, c.poly_p, ptr(Y), ptr(B),
             ptr(geo), stream(dev))
        self._Y = Y
        self._dY = torch.empty(E, 9, device=dev)
        with torch.enable_grad():
            Bl = B.requires_grad_(True)
            Ws = _RadialNet.apply(Bl, self)
            # node features as planes [N (2l + 1), mult]; l = 1, 2 start at exact zeros (None)
            x = [ops.gather_cat([(self.w["embed"], self._elem)]), None, None]
            for L in range(c.num_layers):
                h, sc0, sc1, sc2 = _NodeIn.apply(x[0], x[1], x[2], self, L)
                m = _Conv.apply(h, Ws[L], self, batch, L)
                o = _PlanarOut.apply(m, self, L)
                x = list(_Gate.apply(*o, sc0, sc1, sc2))
            energy = _Readout.apply(x[0], self)
            (dB,) = torch.autograd.grad(energy, Bl, grad_outputs=self._one)
        g = torch.empty(E, 3, device=dev)
        call("fmd_nequip_edge_basis_bwd", ptr(geo), ptr(self._dY), ptr(dB.contiguous()), ptr(override), n_real_edges,
             E, c.r_max, c.num_bessel, c.poly_p, ptr(g), stream(dev))
        forces = torch.empty(N, 3, device=dev)
        call("fmd_edge_forces", ptr(g), ptr(batch.edge_index), ptr(batch.recv_off), ptr(batch.send_off),
             ptr(batch.send_perm), N, ptr(forces), stream(dev))
        return energy.detach().reshape(1), forces

    energy_forces_fused = energy_forces


__all__ = ["NequIPConfig", "NequIPModel", "coupling_table", "gate", "init_weights", "PATHS"]
