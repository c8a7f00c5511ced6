"""The bundled MatRIS potential (energy, forces, stress) on this library's kernels.

The model of fastmd/models/matris/model.py:99 (``MatRIS``, forward :293, blocks
interaction_block.py:882, readout readout.py:16/:143) evaluated on a graph from this build's
builders (``FixedCapacityGraphBuilder`` with a line graph, the reference's fixed-capacity
``radius_graph_view``) or from arrays (any directed edge list with its bond pairing and triplets,
e.g. the reference's legacy CPU graph). Weights load from a MatRIS ``state_dict`` under the
reference's own key names (``matris_params.parameter_shapes``).

Execution: every contraction runs in ``fmd_gemm_tf32x3`` (tcgen05, FP32 accuracy) with the fused
SiLU epilogues, the first layer of every gated MLP as the decomposed indexed projection (the GEMM on
the source rows, one per gathered source with its parts' weight blocks stacked, and the
gather-add-SiLU epilogue on the edge rows, ``fmd_gather_add_silu``), the gated LayerNorm (+ residual) in ``fmd_gated_ln``, the channel
softmax attention in the paired CSR segment attention, the refinement sums in the CSR segment sum,
the bond maps in ``fmd_pair_aggregate``, the residuals in ``fmd_residual_add``; the geometry, the
radial and three-body bases and the force/virial reduction in ``fmd_matris_*``. The energy is
differentiated by autograd over those kernels with respect to the bond lengths and the edge unit
vectors only; ``fmd_matris_forces`` turns those two gradients into forces and the stress (no
autograd through positions, no strain leaf). Everything is capturable in a CUDA graph; tensors live
on a CUDA device (there is no CPU path).
"""
from __future__ import annotations

import numpy as np
import torch
from torch import Tensor
from torch.autograd import Function

from . import _lib, wide_gemm
from ._lib import FmdCatPart, call, ptr, stream
from .decomposed_indexed_cat_silu_linear import _GatherAddSilu
from .dispatch import OpDispatcher, _attention_csr, _directed_pair_index
from .gated_ln import fused_gated_ln, fused_gated_ln_residual
from .matris_params import MATRIS_10M, MatRISConfig, parameter_shapes, seeded_parameters
from .ops import csr_offsets, csr_scope, gather_cat, segment_csr

GPA = 160.21766208  # eV/A^3 -> GPa (readout.py:226)
_ACT_SILU_GRAD, _ACT_INPUT_SILU = 2, 16
_PAD = 8  # basis rows padded to 8 columns (16-byte rows for the projections)


# ----------------------------------------------------------------------------- autograd pieces


class _Bessel(Function):
    """(rbf_atom, rbf_line) [U, 8] of the bond lengths [U] (``fmd_matris_bessel``)."""

    @staticmethod
    def forward(ctx, bond_len, freq_atom, freq_line, consts):
        n_basis, rc_a, rc_l, p = consts
        U = bond_len.shape[0]
        dev = bond_len.device
        rbf_a = torch.empty((U, _PAD), device=dev)
        rbf_l = torch.empty((U, _PAD), device=dev)
        call("fmd_matris_bessel", ptr(bond_len), None, U, U, ptr(freq_atom), ptr(freq_line), n_basis, rc_a, rc_l, p,
             ptr(rbf_a), ptr(rbf_l), _PAD, stream(dev))
        ctx.save_for_backward(bond_len, freq_atom, freq_line)
        ctx.consts = consts
        return rbf_a, rbf_l

    @staticmethod
    def backward(ctx, grad_a, grad_l):
        bond_len, freq_atom, freq_line = ctx.saved_tensors
        n_basis, rc_a, rc_l, p = ctx.consts
        U = bond_len.shape[0]
        dev = bond_len.device
        grad_a = torch.zeros((U, _PAD), device=dev) if grad_a is None else grad_a.contiguous()
        grad_l = torch.zeros((U, _PAD), device=dev) if grad_l is None else grad_l.contiguous()
        grad_len = torch.empty(U, device=dev)
        call("fmd_matris_bessel_bwd", ptr(bond_len), None, U, U, ptr(freq_atom), ptr(freq_line), n_basis, rc_a, rc_l,
             p, ptr(grad_a), ptr(grad_l), _PAD, ptr(grad_len), stream(dev))
        return grad_len, None, None, None


class _ThreeBody(Function):
    """Fourier basis [T, 8] of the triplet angles from the edge unit vectors (``fmd_matris_threebody``)."""

    @staticmethod
    def forward(ctx, unit, graph, freq):
        T, E = graph.line_graph.shape[0], unit.shape[0]
        dev = unit.device
        basis = torch.empty((T, _PAD), device=dev)
        call("fmd_matris_threebody", ptr(unit), ptr(graph.line_graph), T, E, ptr(freq), freq.numel(), ptr(basis),
             _PAD, ptr(_lib.flags_word(dev)), stream(dev))
        ctx.save_for_backward(unit, freq)
        ctx.graph = graph
        return basis

    @staticmethod
    def backward(ctx, grad_basis):
        unit, freq = ctx.saved_tensors
        g = ctx.graph
        T, E = g.line_graph.shape[0], unit.shape[0]
        dev = unit.device
        grad_cos = torch.empty(max(T, 1), device=dev)
        grad_unit = torch.zeros((E, 3), device=dev)
        p1, o1, p2, o2 = g.line_csr
        call("fmd_matris_threebody_bwd", ptr(unit), ptr(g.line_graph), T, E, ptr(freq), freq.numel(),
             ptr(grad_basis.contiguous()), _PAD, ptr(g.pair_index), g.n_bonds, ptr(p1), ptr(o1), ptr(p2), ptr(o2),
             ptr(grad_cos), ptr(grad_unit), stream(dev))
        return grad_unit, None, None


def _gemm_f32(a: Tensor, w: Tensor, transposed: bool, bias=None, a_pre=None, act: int = 0, y_pre=None) -> Tensor:
    """IEEE FP32 ``a' @ B (+ bias)`` on the CUDA cores (``fmd_gemm_f32``): ``B = w^T`` (or ``w`` when
    ``transposed``), ``a' = a * silu'(a_pre)`` when ``a_pre`` is given, SiLU output with ``act = 1`` (the
    pre-activation into ``y_pre``)."""
    m, k = a.shape
    n = w.shape[1] if transposed else w.shape[0]
    y = torch.empty((m, n), device=a.device)
    if m:
        call("fmd_gemm_f32", ptr(a), a.stride(0), ptr(a_pre), a_pre.stride(0) if a_pre is not None else 0, ptr(w),
             w.stride(0), int(not transposed), ptr(bias), ptr(y), n, ptr(y_pre), n if y_pre is not None else 0, m, n,
             k, act, 0, stream(a.device))
    return y


class _PackedGatherAddSilu(Function):
    """``(silu(pre[:, :H]), silu(pre[:, H:]))`` with ``pre = p0 + P_s[:, c : c + 2H][index] + ... + bias``
    where several gathered parts may be column blocks of ONE projection ``P_s`` (a gathered source's
    first-layer weights of all its parts stacked: one GEMM instead of one per part). The backward writes
    each part's CSR row sums into its column block of ``grad_P`` directly (``fmd_gather_rows_bwd``), so a
    shared source gets one gradient tensor and one input-gradient GEMM."""

    @staticmethod
    def forward(ctx, p0, bias, n_sources, blocks, *args):
        # args: the n_sources projections, then one index per part; blocks: (source, column offset) per part
        sources, indices = args[:n_sources], args[n_sources:]
        rows, width = p0.shape
        h = width // 2
        dev = p0.device
        pre = torch.empty((rows, width), device=dev)
        core = torch.empty((rows, h), device=dev)
        gate = torch.empty((rows, h), device=dev)
        parts = (FmdCatPart * len(blocks))()
        for k, ((src, col), idx) in enumerate(zip(blocks, indices)):
            P = sources[src]
            parts[k].src, parts[k].index, parts[k].ld, parts[k].n_src, parts[k].width = (
                P.data_ptr() + 4 * col, ptr(idx), P.stride(0), P.shape[0], width)
        call("fmd_gather_add_silu", ptr(p0), p0.stride(0), parts, len(blocks), ptr(bias), rows, h, ptr(pre),
             ptr(core), ptr(gate), ptr(_lib.flags_word(dev)), stream(dev))
        ctx.save_for_backward(pre, *indices)
        ctx.shapes = [tuple(P.shape) for P in sources]
        ctx.blocks = blocks
        return core, gate

    @staticmethod
    def backward(ctx, grad_core, grad_gate):
        pre, *indices = ctx.saved_tensors
        rows, width = pre.shape
        h = width // 2
        dev = pre.device
        s = stream(dev)
        grad_core = torch.zeros((rows, h), device=dev) if grad_core is None else grad_core.contiguous()
        grad_gate = torch.zeros((rows, h), device=dev) if grad_gate is None else grad_gate.contiguous()
        grad_p0 = torch.empty((rows, width), device=dev)
        call("fmd_silu_pair_bwd", ptr(grad_core), ptr(grad_gate), ptr(pre), rows, h, ptr(grad_p0), width, s)
        grads = [torch.empty(shape, device=dev) for shape in ctx.shapes]
        for (src, col), idx in zip(ctx.blocks, indices):
            n_src, ld = ctx.shapes[src]
            perm, off = segment_csr(idx, n_src)
            if n_src:
                # long runs (e.g. an atom's triplets): eight warps per source row
                name = "fmd_gather_rows_bwd_long" if rows >= 64 * n_src else "fmd_gather_rows_bwd"
                call(name, ptr(grad_p0), width, 0, width, ptr(perm), ptr(off), n_src,
                     grads[src].data_ptr() + 4 * col, ld, 0, s)
        return (grad_p0, None, None, None, *grads, *([None] * len(indices)))


class _LineEnvelope(Function):
    """env [T, C] = base[u2] * base[u1] over the triplets (``fmd_matris_line_envelope``), the backward a CSR fold
    per bond (``fmd_matris_line_envelope_bwd``)."""

    @staticmethod
    def forward(ctx, base, graph):
        T, C = graph.line_graph.shape[0], base.shape[1]
        base = base.contiguous()
        env = torch.empty((T, C), device=base.device)
        call("fmd_matris_line_envelope", ptr(base), base.stride(0), ptr(graph.line_graph), T, graph.n_bonds, C,
             ptr(env), C, ptr(_lib.flags_word(base.device)), stream(base.device))
        ctx.save_for_backward(base)
        ctx.graph = graph
        return env

    @staticmethod
    def backward(ctx, grad):
        (base,) = ctx.saved_tensors
        g = ctx.graph
        grad = grad.contiguous()
        out = torch.empty_like(base)
        p1, o1, p2, o2 = g.line_csr
        call("fmd_matris_line_envelope_bwd", ptr(base), base.stride(0), ptr(g.line_graph), g.n_bonds, base.shape[1],
             ptr(grad), grad.stride(0), ptr(p1), ptr(o1), ptr(p2), ptr(o2), ptr(out), out.stride(0),
             stream(base.device))
        return out, None


class _SiluChain(Function):
    """``L_n(silu(... silu(L_1(x))))`` of frozen linears ``L_k(x) = x W_k^T (+ b_k)``.

    ``tf32x3``: on the tensor cores, each SiLU applied to the next layer's operand
    (``FMD_ACT_INPUT_SILU``), the backward forming ``(dY W_k) * silu'(h)`` in the GEMM epilogue
    (``FMD_ACT_SILU_GRAD``). ``ieee``: on the CUDA cores, each hidden layer writing its SiLU output and
    its pre-activation, the backward multiplying the next operand by ``silu'(h)`` as it loads it."""

    @staticmethod
    def forward(ctx, x, precision, *layers):
        n = len(layers) // 2
        hs = []
        h = x
        for k in range(n):
            w, b = layers[2 * k], layers[2 * k + 1]
            if precision == "tf32x3":
                h = wide_gemm._launch(h if k == 0 else hs[-1], w, False, "tf32x3", b, act=_ACT_INPUT_SILU if k else 0)
                hs.append(h)
            elif k + 1 < n:
                pre = torch.empty((h.shape[0], w.shape[0]), device=h.device)
                h = _gemm_f32(h, w, False, b, act=1, y_pre=pre)
                hs.append(pre)
            else:
                hs.append(_gemm_f32(h, w, False, b))
        ctx.save_for_backward(*hs[:-1], *layers[0::2])
        ctx.n, ctx.precision = n, precision
        return hs[-1]

    @staticmethod
    def backward(ctx, grad):
        saved = ctx.saved_tensors
        n = ctx.n
        hs, ws = saved[:n - 1], saved[n - 1:]
        g = grad.contiguous()
        if ctx.precision == "tf32x3":
            for k in range(n - 1, 0, -1):
                g = wide_gemm._launch(g, ws[k], True, "tf32x3", c=hs[k - 1], act=_ACT_SILU_GRAD)
            g = wide_gemm._launch(g, ws[0], True, "tf32x3")
        else:
            g = _gemm_f32(g, ws[n - 1], True)
            for k in range(n - 2, -1, -1):
                g = _gemm_f32(g, ws[k], True, a_pre=hs[k])
        return (g, None, *([None] * (2 * n)))


def _silu_chain(x: Tensor, layers: list, precision: str) -> Tensor:
    flat = []
    for w, b in layers:
        flat.extend([w, b])
    return _SiluChain.apply(x, precision, *flat)


# ----------------------------------------------------------------------------- graph


class MatRISGraph:
    """One evaluation's graph on the device: edges [E, 2] (centre, neighbour) with images, the bond pairing
    ``d2u`` [E] / ``u2d`` [U] and triplets [T, 5], plus the CSRs and dispatcher state derived from them
    (rebuilt per graph; capture-safe)."""

    def __init__(self, positions: Tensor, cell: Tensor, species: Tensor, edge_index: Tensor, edge_image: Tensor,
                 d2u: Tensor, u2d: Tensor, line_graph: Tensor, n_real: int, *, centre_sorted: bool):
        _lib.require_cuda(positions, cell, species, edge_index, edge_image, d2u, u2d, line_graph)
        dev = positions.device
        self.device = dev
        self.positions = positions.to(torch.float32).contiguous()
        self.cell = cell.to(device=dev, dtype=torch.float32).reshape(3, 3).contiguous()
        self.species = species.to(torch.int64).contiguous()
        self.element = (self.species - 1).contiguous()  # embedding row of each atom (Z - 1)
        self.edge_index = edge_index.to(torch.int32).contiguous()
        self.edge_image = edge_image.to(torch.float32).contiguous()
        self.d2u = d2u.to(torch.int32).contiguous()
        self.u2d = u2d.to(torch.int32).contiguous()
        self.line_graph = line_graph.to(torch.int32).reshape(-1, 5).contiguous()
        self.n_atoms = self.positions.shape[0]
        self.n_edges = self.edge_index.shape[0]
        self.n_bonds = self.u2d.shape[0]
        self.n_triplets = self.line_graph.shape[0]
        self.n_real = int(n_real)
        if self.n_edges != 2 * self.n_bonds:
            raise ValueError(f"{self.n_edges} directed edges for {self.n_bonds} bonds (need E == 2U)")
        lg = self.line_graph.to(torch.int64)
        self.centre = self.edge_index[:, 0].to(torch.int64)
        self.neighbour = self.edge_index[:, 1].to(torch.int64)
        self.u2d64 = self.u2d.to(torch.int64)
        self.t_atom, self.t_u1, self.t_u2 = lg[:, 0].contiguous(), lg[:, 1].contiguous(), lg[:, 3].contiguous()
        self.ops = OpDispatcher(identity_target_csr=("atom",) if centre_sorted else ())
        self.atom = {"source_index": self.neighbour, "target_index": self.centre, "num_segment": self.n_atoms,
                     "num_undirected": self.n_bonds, "_topology_graph_kind": "atom", "_ops": self.ops}
        if centre_sorted:
            self.atom["_target_segment_attention_offsets"] = csr_offsets(self.centre, self.n_atoms)
        self.line = {"source_index": self.t_u2, "target_index": self.t_u1, "num_segment": self.n_bonds,
                     "num_undirected": self.n_bonds, "_topology_graph_kind": "line", "_ops": self.ops}
        self.ops.prepare_segment_csr(self.atom, self.n_atoms)
        self.ops.prepare_segment_csr(self.line, self.n_bonds)
        self.pair_index = _directed_pair_index(self.atom, self.d2u.to(torch.int64))
        p1, o1, _ = _attention_csr(self.line, "target", self.t_u1, self.n_bonds, False)
        p2, o2, _ = _attention_csr(self.line, "source", self.t_u2, self.n_bonds, False)
        self.line_csr = (p1, o1, p2, o2)
        recv_perm, recv_off, identity = _attention_csr(self.atom, "target", self.centre, self.n_atoms, centre_sorted)
        self.recv = (None if identity else recv_perm, recv_off)
        self.send = _attention_csr(self.atom, "source", self.neighbour, self.n_atoms, False)[:2]
        # a line-graph layer acts only when some triplet is centred on a real atom (interaction_block.py:1044)
        self.real_line = (self.t_atom < self.n_real).any()

    @classmethod
    def from_arrays(cls, positions, cell, numbers, edge_index, edge_image, d2u, u2d, line_graph, *, n_real=None,
                    device="cuda") -> "MatRISGraph":
        """A graph from host arrays (e.g. the reference's legacy CPU graph): edges in any order."""
        ei = np.asarray(edge_index, np.int64).reshape(-1, 2)
        sorted_centres = bool(np.all(np.diff(ei[:, 0]) >= 0))
        dev = torch.device(device)
        t = lambda a, dt: torch.as_tensor(np.asarray(a), dtype=dt).to(dev)  # noqa: E731
        n = np.asarray(positions).shape[0]
        return cls(t(positions, torch.float32), t(cell, torch.float32), t(numbers, torch.int64),
                   t(ei, torch.int32), t(edge_image, torch.float32), t(d2u, torch.int32), t(u2d, torch.int32),
                   t(np.asarray(line_graph).reshape(-1, 5), torch.int32), n if n_real is None else n_real,
                   centre_sorted=sorted_centres)

    @classmethod
    def from_batch(cls, batch) -> "MatRISGraph":
        """The graph of a ``FixedCapacityGraphBuilder`` batch with a line graph (capacity rows included: padding
        sits on sink atoms past ``n_real``, which the energy leaves out)."""
        if batch.line_graph is None:
            raise ValueError("MatRIS needs a builder with a line graph (line_graph_cutoff, t_capacity)")
        return cls(batch.positions, batch.cell, batch.species, batch.edge_index, batch.edge_image,
                   batch.directed2undirected, batch.undirected2directed, batch.line_graph, batch.n_real,
                   centre_sorted=True)


# ----------------------------------------------------------------------------- model


class _Gated:
    """A GatedMLP's frozen weights (functions.py:395): the first layers of core and gate stacked
    ``[2C, K]`` and cut into ``K / C`` column blocks (one per concatenated part), the second layers,
    their biases (added inside the gated LayerNorm) and the two LayerNorms."""

    def __init__(self, p: dict, key: str, parts: int, C: int, precision: str):
        self.precision = precision
        w0 = torch.cat([p[f"{key}.mlp_core.layers.0.weight"], p[f"{key}.mlp_gate.layers.0.weight"]], 0)
        self.w0 = w0.contiguous()
        self.parts = tuple(w0[:, i * C:(i + 1) * C].contiguous() for i in range(parts))
        # the gathered parts' first-layer blocks stacked per gathered source (one projection per source):
        # cat3 [A | X[a] | X[b]] -> X (W_a; W_b); cat4 [A | Y[a] | X[b] | X[c]] -> Y W_a, X (W_b; W_c)
        blocks = self.parts[1:]
        self.sources = ((torch.cat(blocks, 0).contiguous(),) if parts == 3 else
                        (blocks[0], torch.cat(blocks[1:], 0).contiguous()))
        self.b0 = torch.cat([p[f"{key}.mlp_core.layers.0.bias"], p[f"{key}.mlp_gate.layers.0.bias"]]).contiguous()
        self.w3c, self.b3c = p[f"{key}.mlp_core.layers.3.weight"], p[f"{key}.mlp_core.layers.3.bias"]
        self.w3g, self.b3g = p[f"{key}.mlp_gate.layers.3.weight"], p[f"{key}.mlp_gate.layers.3.bias"]
        self.ln = (p[f"{key}.core_norm.weight"], p[f"{key}.core_norm.bias"], p[f"{key}.gate_norm.weight"],
                   p[f"{key}.gate_norm.bias"])

    def __call__(self, core: Tensor, gate: Tensor, residual: Tensor | None = None, res_weight: Tensor | None = None):
        core_x = wide_gemm.linear(core, self.w3c, precision=self.precision)
        gate_x = wide_gemm.linear(gate, self.w3g, precision=self.precision)
        if residual is None:
            return fused_gated_ln(core_x, gate_x, *self.ln, 1e-5, 1e-5, core_lb=self.b3c, gate_lb=self.b3g)
        return fused_gated_ln_residual(core_x, gate_x, *self.ln, residual, res_weight, 1e-5, 1e-5,
                                       core_lb=self.b3c, gate_lb=self.b3g)


class MatRISModel:
    """MatRIS on one CUDA device with frozen weights.

    ``params``: a MatRIS ``state_dict`` (reference key names; tensors or arrays), default the seeded
    random weights of ``matris_params.seeded_parameters(config, seed)``.
    ``energy_forces_stress(graph)`` -> (energy [1] float64, forces [n_real, 3] float32,
    stress [3, 3] float32 GPa); ``graph`` is a ``MatRISGraph`` or a builder batch.
    """

    def __init__(self, config: MatRISConfig = MATRIS_10M, params: dict | None = None, *, seed: int = 0,
                 device="cuda", precision: str = "tf32x3"):
        if precision not in wide_gemm.PRECISIONS:
            raise ValueError(f"precision must be one of {wide_gemm.PRECISIONS}, got {precision!r}")
        self.config = config
        self.precision = precision
        self.device = torch.device(device)
        _lib.require_cuda(torch.empty(0, device=self.device))
        if params is None:
            params = seeded_parameters(config, seed)
        expected = {k: s for k, s, _ in parameter_shapes(config)}
        missing = set(expected) - set(params)
        if missing:
            raise KeyError(f"MatRIS parameters missing: {sorted(missing)[:5]} ...")
        p = {k: torch.as_tensor(np.asarray(params[k].detach().cpu() if isinstance(params[k], Tensor) else params[k]),
                                dtype=torch.float32).to(self.device).contiguous() for k in expected}
        for k, shape in expected.items():
            if tuple(p[k].shape) != tuple(shape):
                raise ValueError(f"{k}: shape {tuple(p[k].shape)}, expected {shape}")
        self.params = p
        C, R = config.node_dim, config.num_radial

        def padded(w, width=_PAD):
            out = torch.zeros((w.shape[0], width), device=self.device)
            out[:, :w.shape[1]] = w
            return out

        # atom embedding: a per-element table (positions do not enter it)
        table = p["atom_embedding.embedding.weight"] @ p["atom_embedding.atom_swish_layer.linear.weight"].T
        self.atom_table = torch.nn.functional.silu(table).contiguous()
        self.freq_atom = p["edge_embedding.pairwise_rbf_expansion.frequencies"]
        self.freq_line = p["edge_embedding.threebody_rbf_expansion.frequencies"]
        self.freq_angle = p["three_body_embedding.expansion.frequencies"]
        self.bessel_consts = (R, float(config.pairwise_cutoff), float(config.three_body_cutoff),
                              float(config.envelope_exponent))
        self.edge_w1 = padded(p["edge_embedding.edge_linear1.weight"])
        self.edge_w2 = p["edge_embedding.edge_linear2.weight"]
        self.edge_ln = (p["edge_embedding.edge_init_norm.weight"], p["edge_embedding.edge_init_norm.bias"])
        self.edge_ws = p["edge_embedding.swish_layer.linear.weight"]
        self.angle_w = padded(p["three_body_embedding.angle_embedding.weight"])
        self.angle_ws = p["three_body_embedding.swish_layer.linear.weight"]
        self.blocks = []
        for b in range(config.num_layers):
            blk = {}
            for graph in ("atom", "line"):
                key = f"interaction_block.{b}.attn_block_{graph}_graph"
                blk[f"attn_{graph}"] = dict(
                    edge=_Gated(p, f"{key}.edge_nonlinear_update", 3, C, precision),
                    node=_Gated(p, f"{key}.node_nonlinear_update", 3, C, precision),
                    logits=torch.cat([p[f"{key}.source_weight_linear.weight"],
                                      p[f"{key}.target_weight_linear.weight"]], 0).contiguous(),
                    node_res=p[f"{key}.node_res_weight"].reshape(-1), edge_res=p[f"{key}.edge_res_weight"].reshape(-1))
                key = f"interaction_block.{b}.refine_block_{graph}_graph"
                blk[f"refine_{graph}"] = dict(
                    edge=_Gated(p, f"{key}.edge_nonlinear_update", 3 if graph == "atom" else 4, C, precision),
                    node_ffn=[(p[f"{key}.node_FFN.layers.0.weight"], None), (p[f"{key}.node_FFN.layers.3.weight"], None)],
                    edge_ffn=[(p[f"{key}.edge_FFN.layers.0.weight"], None), (p[f"{key}.edge_FFN.layers.3.weight"], None)],
                    envelope=padded(p[f"{key}.learnable_envelope.weight"]),
                    node_res=p[f"{key}.node_res_weight"].reshape(-1), edge_res=p[f"{key}.edge_res_weight"].reshape(-1))
            self.blocks.append(blk)
        self.readout_ln = (p["readout_norm.weight"], p["readout_norm.bias"])
        widths = [C, *config.energy_hidden, 1]
        head = []
        for i in range(len(widths) - 1):
            w, bias = p[f"energy_head.energy_head.layers.{3 * i}.weight"], p[f"energy_head.energy_head.layers.{3 * i}.bias"]
            if i == len(widths) - 2:  # the 1-wide output padded to 4 columns (16-byte rows)
                w4 = torch.zeros((4, w.shape[1]), device=self.device)
                w4[:1] = w
                b4 = torch.zeros(4, device=self.device)
                b4[:1] = bias
                w, bias = w4, b4
            head.append((w.contiguous(), bias.contiguous()))
        self.head = head

    # ------------------------------------------------------------------ layers

    def _first_layer(self, gm: _Gated, aligned: Tensor, gathered: list) -> tuple[Tensor, Tensor]:
        """The SiLU halves of ``[aligned | gathered rows...] @ W0^T + b0`` by parts: ``aligned`` projected row
        by row, each gathered source projected once on its own rows (all its parts' weight blocks stacked)
        and its rows gathered and added in the epilogue (``gathered``: (source, [index per part]))."""
        p0 = wide_gemm.linear(aligned, gm.parts[0], precision=self.precision)
        sources, blocks, indices = [], [], []
        width = gm.parts[0].shape[0]
        for n, ((x, idxs), w) in enumerate(zip(gathered, gm.sources)):
            sources.append(wide_gemm.linear(x, w, precision=self.precision))
            for j, idx in enumerate(idxs):
                blocks.append((n, j * width))
                indices.append(idx)
        return _PackedGatherAddSilu.apply(p0, gm.b0, len(sources), tuple(blocks), *sources, *indices)

    def _attention(self, layer: dict, nodes: Tensor, edges: Tensor, g: MatRISGraph, graph: dict, kind: str):
        """Graph_Attention_Layer (interaction_block.py:291-481): returns (nodes', edges')."""
        ops = graph["_ops"]
        target, source, n_nodes = graph["target_index"], graph["source_index"], graph["num_segment"]
        rows = ops.pair_expand(edges, g.d2u, graph) if kind == "atom" else edges
        gm = layer["edge"]
        core, gate = self._first_layer(gm, rows, [(nodes, [target, source])])
        msg = gm(core, gate)
        logits = wide_gemm.linear(rows, layer["logits"], precision=self.precision)
        C = edges.shape[1]
        att_s, att_t = ops.segment_attention(logits[:, :C], msg, source, logits[:, C:], msg, target, n_nodes, graph)
        nm = layer["node"]
        pre = wide_gemm.linear(gather_cat([(nodes, None), (att_t, None), (att_s, None)]), nm.w0,
                               precision=self.precision)
        n_core, n_gate = _GatherAddSilu.apply(pre, nm.b0, 0)
        new_nodes = nm(n_core, n_gate, nodes, layer["node_res"])
        m = ops.pair_average(msg, g.d2u, graph) if kind == "atom" else msg
        return new_nodes, ops.residual(m, edges, layer["edge_res"])

    def _refine_atom(self, layer: dict, nodes: Tensor, bonds: Tensor, rbf_atom: Tensor, g: MatRISGraph,
                     edge_update: bool):
        """Refinement on the atom graph (interaction_block.py:580-848)."""
        ops, graph = g.ops, g.atom
        rows = ops.pair_expand(bonds, g.d2u, graph)
        env = ops.pair_expand(wide_gemm.linear(rbf_atom, layer["envelope"], precision=self.precision), g.d2u,
                              graph)
        gm = layer["edge"]
        core, gate = self._first_layer(gm, rows, [(nodes, [g.centre, g.neighbour])])
        raw = gm(core, gate)
        red = ops.segment_sum_graph(raw, g.centre, g.n_atoms, graph, "target", weight=env)
        new_nodes = ops.residual(_silu_chain(red, layer["node_ffn"], self.precision), nodes, layer["node_res"])
        if not edge_update:
            return new_nodes, bonds
        delta = ops.pair_average(_silu_chain(raw, layer["edge_ffn"], self.precision), g.d2u, graph)
        return new_nodes, ops.residual(delta, bonds, layer["edge_res"])

    def _refine_line(self, layer: dict, bonds: Tensor, trips: Tensor, atoms: Tensor, rbf_line: Tensor,
                     g: MatRISGraph, edge_update: bool):
        """Refinement on the line graph (interaction_block.py:580-848): bonds are its nodes."""
        ops, graph = g.ops, g.line
        base = wide_gemm.linear(rbf_line, layer["envelope"], precision=self.precision)
        env = _LineEnvelope.apply(base, g)
        gm = layer["edge"]
        core, gate = self._first_layer(gm, trips, [(atoms, [g.t_atom]), (bonds, [g.t_u1, g.t_u2])])
        raw = gm(core, gate)
        red = ops.segment_sum_graph(raw, g.t_u1, g.n_bonds, graph, "target", weight=env)
        new_bonds = ops.residual(_silu_chain(red, layer["node_ffn"], self.precision), bonds, layer["node_res"])
        if not edge_update:
            return new_bonds, trips
        return new_bonds, ops.residual(_silu_chain(raw, layer["edge_ffn"], self.precision), trips, layer["edge_res"])

    # ------------------------------------------------------------------ evaluation

    def _graph(self, graph) -> MatRISGraph:
        return graph if isinstance(graph, MatRISGraph) else MatRISGraph.from_batch(graph)

    # ------------------------------------------------------------------ the MD drivers' model interface

    @property
    def cutoff(self) -> float:
        """The atom-graph cutoff (A)."""
        return float(self.config.pairwise_cutoff)

    def builder_options(self, positions, cell, n_atoms: int, replicas: int = 1) -> dict:
        """``FixedCapacityGraphBuilder`` arguments for this model: the line graph within the three-body cutoff,
        sink padding with 4 sink atoms per replica, and capacities from one system's ragged graph at
        ``positions`` (pairs x 1.08 rounded up to 32, triplets x 1.15 rounded up to 256; times the replica
        count). One host read (set-up only)."""
        from .graph import neighbor_list

        pos = torch.as_tensor(np.asarray(positions)[:n_atoms], dtype=torch.float32).to(self.device)
        centre, _, _, dist = neighbor_list(pos, torch.as_tensor(np.asarray(cell), dtype=torch.float32), self.cutoff)
        centre, dist = centre.cpu().numpy(), dist.cpu().numpy()
        pairs = (centre.shape[0] + 1) // 2
        short = np.bincount(centre[dist < np.float32(self.config.three_body_cutoff)], minlength=n_atoms)
        triplets = int((short * (short - 1)).sum())
        u_cap = int(np.ceil(max(pairs * 1.08, pairs + 32) / 32.0)) * 32
        t_cap = int(np.ceil(max(triplets * 1.15, triplets + 256) / 256.0)) * 256
        return dict(u_capacity=u_cap * replicas, t_capacity=t_cap * replicas, n_dummy=4 * replicas,
                    line_graph_cutoff=float(self.config.three_body_cutoff))

    def prepare(self, batch) -> None:
        """Nothing to prepare: the graph-derived state is rebuilt inside every evaluation."""

    def energy_forces(self, batch, n_systems: int = 1):
        """(energies [n_systems] float64, forces [n_real, 3] float32) of a builder batch whose real atoms are
        ``n_systems`` equal-sized systems (a replica union)."""
        energy, forces, _ = self.energy_forces_stress(batch, stress=False, n_systems=n_systems)
        return energy, forces

    energy_forces_fused = energy_forces

    def energy_forces_stress(self, graph, *, forces: bool = True, stress: bool = True, n_systems: int = 1):
        """(energies [n_systems] float64, forces [n_real, 3] float32, stress [3, 3] float32 GPa of the whole
        graph) of ``graph``; forces and stress are None when not asked for. Each index tensor of the graph is
        sorted into its CSR once per call (``ops.csr_scope``)."""
        with csr_scope():
            return self._evaluate(graph, forces, stress, int(n_systems))

    def _evaluate(self, graph, forces: bool, stress: bool, n_systems: int):
        g = self._graph(graph)
        dev = g.device
        s = stream(dev)
        length = torch.empty(g.n_edges, device=dev)
        unit = torch.empty((g.n_edges, 3), device=dev)
        call("fmd_matris_geometry", ptr(g.positions), ptr(g.cell), ptr(g.edge_index), ptr(g.edge_image), g.n_edges,
             g.n_atoms, ptr(length), ptr(unit), ptr(_lib.flags_word(dev)), s)
        bond_len = length.index_select(0, g.u2d64)
        need_grad = forces or stress
        if need_grad:
            bond_len.requires_grad_(True)
            unit.requires_grad_(True)
        with torch.set_grad_enabled(need_grad):
            energy = self._energy(g, bond_len, unit, n_systems)
        if not need_grad:
            return energy.detach(), None, None
        grad_len, grad_unit = torch.autograd.grad(energy.sum(), [bond_len, unit], allow_unused=True)
        out_forces = torch.empty((g.n_atoms, 3), device=dev)
        rows = torch.empty((g.n_atoms, 9), dtype=torch.float64, device=dev) if stress else None
        out_stress = torch.empty(9, device=dev) if stress else None
        recv_perm, recv_off = g.recv
        send_perm, send_off = g.send
        call("fmd_matris_forces", ptr(length), ptr(unit.detach()), ptr(grad_len), ptr(grad_unit), ptr(g.d2u),
             ptr(g.u2d), ptr(g.edge_index), g.n_edges, g.n_bonds, g.n_atoms, ptr(recv_perm), ptr(recv_off),
             ptr(send_perm), ptr(send_off), ptr(g.cell), GPA, ptr(out_forces), ptr(rows), ptr(out_stress), None, s)
        return (energy.detach(), out_forces[:g.n_real] if forces else None,
                out_stress.reshape(3, 3) if stress else None)

    def energy(self, graph) -> Tensor:
        return self.energy_forces_stress(graph, forces=False, stress=False)[0]

    def _energy(self, g: MatRISGraph, bond_len: Tensor, unit: Tensor, n_systems: int) -> Tensor:
        C = self.config.node_dim
        rbf_atom, rbf_line = _Bessel.apply(bond_len, self.freq_atom, self.freq_line, self.bessel_consts)
        # embeddings (feature_embed.py:89-247, 373-475)
        nodes = gather_cat([(self.atom_table, g.element)])
        prec = self.precision
        bonds = wide_gemm.linear(wide_gemm.linear(rbf_atom, self.edge_w1, precision=prec), self.edge_w2,
                                 precision=prec)
        bonds = torch.nn.functional.layer_norm(bonds, (C,), *self.edge_ln, 1e-5)
        bonds = torch.nn.functional.silu(wide_gemm.linear(bonds, self.edge_ws, precision=self.precision))
        basis = _ThreeBody.apply(unit, g, self.freq_angle)
        trips = wide_gemm.linear(wide_gemm.linear(basis, self.angle_w, precision=prec), self.angle_ws, precision=prec)
        trips = torch.nn.functional.silu(trips)
        last = len(self.blocks) - 1
        for b, blk in enumerate(self.blocks):
            bonds_in = bonds
            new_bonds, trips = self._attention(blk["attn_line"], bonds, trips, g, g.line, "line")
            bonds = torch.where(g.real_line, new_bonds, bonds_in)
            nodes, bonds = self._attention(blk["attn_atom"], nodes, bonds, g, g.atom, "atom")
            new_bonds, trips = self._refine_line(blk["refine_line"], bonds, trips, nodes, rbf_line, g, b < last)
            bonds = torch.where(g.real_line, new_bonds, bonds_in)
            nodes, bonds = self._refine_atom(blk["refine_atom"], nodes, bonds, rbf_atom, g, b < last)
        readout = torch.nn.functional.layer_norm(nodes, (C,), *self.readout_ln, 1e-5)
        per_atom = _silu_chain(readout, self.head, self.precision)[:, 0]
        if g.n_real % n_systems:
            raise ValueError(f"{g.n_real} real atoms do not split into {n_systems} equal systems")
        return per_atom[:g.n_real].double().reshape(n_systems, -1).sum(1)


__all__ = ["MatRISModel", "MatRISGraph"]
