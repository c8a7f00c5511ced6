"""FP64 CPU restatement of the bundled MatRIS potential -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs use this module, as the
checker of the CUDA path (``fastmd_b200.matris``); nothing in the package imports it.

It restates, in plain torch on the CPU, the equations of the reference's MatRIS
(fastmd/models/matris/model.py:293 ``_forward``) as its plain-torch dispatch computes them:

* geometry (processgraph.py:218-233): ``v_e = x[centre] - (x[neighbour] + image_e @ L)``, ``d_e = |v_e|``,
  ``u_e = v_e / d_e``; the undirected lengths are ``d[undirected2directed]``;
* embeddings (feature_embed.py:89-247, 373-475): ``silu(W_s Emb[Z - 1])`` per atom; per bond
  ``silu(W_s LN(W_2 W_1 rbf_6(d)))`` with the Bessel basis ``sqrt(2/rc) sin(f d/rc)/d`` times the polynomial
  envelope (basis_function.py:31-75, 139-209) and learnable frequencies ``f``; per triplet
  ``silu(W_s W_a fourier(theta))`` with ``theta = acos((u_e1 . u_e2)(1 - 1e-6))`` and
  ``fourier = [2^-1/2, sin(k theta), cos(k theta)] / sqrt(pi)`` (basis_function.py:102-136);
* per interaction block (interaction_block.py:991-1130): line-graph attention over the bonds, atom-graph
  attention over the atoms, line-graph refinement, atom-graph refinement;
  - attention (:291-481): ``m = GatedMLP([edge | node[target] | node[source]])``, logits
    ``a_s = W_src edge``, ``a_t = W_tgt edge``, channel-wise softmax of the logits over each node's
    segment (engine/kernels/segment.py:57-94), ``node' = GatedMLP([node | att_t | att_s]) + node * w_n``,
    ``edge' = pair_average(m) + edge * w_e`` (the atom graph averages a bond's two directed rows);
  - refinement (:580-848): ``raw = GatedMLP([edge | (atom[centre] |) node[target] | node[source]])``,
    envelope ``W_env rbf_4.5`` (line graph: the product of the two bonds' envelopes) or ``W_env rbf_6``
    expanded to directed rows (atom graph), ``node' = FFN(sum_target envelope * raw) + node * w_n``,
    ``edge' = pair_average(FFN(raw)) + edge * w_e``;
  - a line-graph layer leaves the bonds unchanged when no triplet touches a real atom (:1044-1099);
* readout (model.py:438-520): ``E = sum_real MLP(LN(node))`` in FP64; forces ``-dE/dx``; stress
  ``dE/d(strain) / V`` in GPa (readout.py:200-230), the strain applied as ``x (1 + e)``, ``L (1 + e)``
  with ``e`` symmetrised (processgraph.py:185-211).

``GatedMLP(x) = silu(LN(MLP_c(x))) * sigmoid(LN(MLP_g(x)))`` with ``MLP = Linear -> SiLU -> Linear``
(functions.py:152-252, 395-513, 1086-1123).

Pinned against the reference model itself run on CPU (tests/golden/matris.npz, made by
tests/golden/make_golden.py): energy, forces and stress of the FP64 evaluation to 1e-10 relative.
"""
from __future__ import annotations

import math

import numpy as np
import torch

GPA = 160.21766208  # eV/A^3 -> GPa, readout.py:226


def _lin(x, p, key, bias=True):
    y = x @ p[key + ".weight"].T
    b = p.get(key + ".bias") if bias else None
    return y if b is None else y + b


def _ln(x, p, key, eps=1e-5):
    mu = x.mean(-1, keepdim=True)
    var = ((x - mu) ** 2).mean(-1, keepdim=True)
    return (x - mu) / torch.sqrt(var + eps) * p[key + ".weight"] + p[key + ".bias"]


def _mlp(x, p, key, n_linear):
    """Linear -> SiLU -> ... -> Linear, the linears at layers 0, 3, 6, ... (dropout slots between)."""
    for i in range(n_linear):
        x = _lin(x, p, f"{key}.layers.{3 * i}")
        if i + 1 < n_linear:
            x = torch.nn.functional.silu(x)
    return x


def _gated(x, p, key):
    core = _ln(_mlp(x, p, key + ".mlp_core", 2), p, key + ".core_norm")
    gate = _ln(_mlp(x, p, key + ".mlp_gate", 2), p, key + ".gate_norm")
    return torch.nn.functional.silu(core) * torch.sigmoid(gate)


def _bessel(d, freq, cutoff, exponent):
    """Bessel basis times the polynomial envelope (basis_function.py:31-75, 185-209), rows [len(d), n]."""
    d = d[:, None]
    x = d / cutoff
    p = float(exponent)
    a, b, c = -(p + 1) * (p + 2) / 2, p * (p + 2), -p * (p + 1) / 2
    env = torch.where(x < 1, 1 + a * x ** p + b * x ** (p + 1) + c * x ** (p + 2), torch.zeros_like(x))
    return env * (math.sqrt(2.0 / cutoff) * torch.sin(freq * x) / d)


def _fourier(theta, freq):
    k = theta[:, None] * freq[None, :]
    const = torch.full_like(theta[:, None], 2 ** -0.5)
    return torch.cat([const, torch.sin(k), torch.cos(k)], dim=1) / math.sqrt(math.pi)


def _softmax_sum(logits, value, segment, n):
    """Channel-wise softmax of ``logits`` over each segment, weighted sum of ``value`` rows."""
    width = logits.shape[1]
    idx = segment[:, None].expand(-1, width)
    peak = torch.full((n, width), -math.inf, dtype=logits.dtype).scatter_reduce(0, idx, logits, "amax",
                                                                                   include_self=True)
    w = torch.exp(logits - peak[segment])
    den = torch.zeros((n, width), dtype=logits.dtype).index_add_(0, segment, w)
    return torch.zeros((n, width), dtype=logits.dtype).index_add_(0, segment, w / den[segment] * value)


def _segment_sum(value, segment, n):
    return torch.zeros((n, value.shape[1]), dtype=value.dtype).index_add_(0, segment, value)


def _pair_average(data, d2u, n_undirected):
    count = torch.zeros(n_undirected, dtype=data.dtype).index_add_(0, d2u, torch.ones_like(d2u, dtype=data.dtype))
    return _segment_sum(data, d2u, n_undirected) / count.clamp(min=1)[:, None]


def energy_forces_stress(params, config, positions, cell, numbers, edge_index, edge_image, d2u, u2d, line_graph,
                         n_real=None, dtype=torch.float64):
    """(E [float], forces [N, 3], stress [3, 3] GPa) as NumPy float64, for one periodic system whose graph
    is given as arrays: ``edge_index`` [E, 2] (centre, neighbour), ``edge_image`` [E, 3] (lattice units),
    ``d2u`` [E], ``u2d`` [U], ``line_graph`` [T, 5] (atom, u1, e1, u2, e2). ``n_real``: atoms past it are
    padding rows (left out of the energy and the real-triplet test)."""
    p = {k: torch.as_tensor(np.asarray(v), dtype=dtype) for k, v in params.items()}
    C = config
    n = positions.shape[0]
    n_real = n if n_real is None else int(n_real)
    ei = torch.as_tensor(np.asarray(edge_index, np.int64))
    centre, neighbour = ei[:, 0], ei[:, 1]
    d2u = torch.as_tensor(np.asarray(d2u, np.int64))
    u2d = torch.as_tensor(np.asarray(u2d, np.int64))
    lg = torch.as_tensor(np.asarray(line_graph, np.int64)).reshape(-1, 5)
    n_u = u2d.shape[0]
    t_atom, t_u1, t_e1, t_u2, t_e2 = lg.unbind(1)

    x0 = torch.as_tensor(np.asarray(positions), dtype=dtype).clone().requires_grad_(True)
    strain = torch.zeros((3, 3), dtype=dtype, requires_grad=True)
    sym = 0.5 * (strain + strain.T)
    lat0 = torch.as_tensor(np.asarray(cell), dtype=dtype).reshape(3, 3)
    x = x0 + x0 @ sym
    lat = lat0 + lat0 @ sym
    vec = x[centre] - (x[neighbour] + torch.as_tensor(np.asarray(edge_image), dtype=dtype) @ lat)
    length = torch.linalg.norm(vec, dim=1)
    unit = vec / length[:, None]

    # embeddings
    z = torch.as_tensor(np.asarray(numbers, np.int64)) - 1
    node = torch.nn.functional.silu(_lin(p["atom_embedding.embedding.weight"][z], p,
                                         "atom_embedding.atom_swish_layer.linear", bias=False))
    ulen = length[u2d]
    rbf_atom = _bessel(ulen, p["edge_embedding.pairwise_rbf_expansion.frequencies"], C.pairwise_cutoff,
                       C.envelope_exponent)
    rbf_line = _bessel(ulen, p["edge_embedding.threebody_rbf_expansion.frequencies"], C.three_body_cutoff,
                       C.envelope_exponent)
    bond = _lin(_lin(rbf_atom, p, "edge_embedding.edge_linear1", False), p, "edge_embedding.edge_linear2", False)
    bond = torch.nn.functional.silu(_lin(_ln(bond, p, "edge_embedding.edge_init_norm"), p,
                                         "edge_embedding.swish_layer.linear", False))
    has_triplets = lg.shape[0] > 0
    if has_triplets:
        cos = (unit[t_e1] * unit[t_e2]).sum(1) * (1 - 1e-6)
        basis = _fourier(torch.acos(cos), p["three_body_embedding.expansion.frequencies"])
        trip = torch.nn.functional.silu(_lin(_lin(basis, p, "three_body_embedding.angle_embedding", False), p,
                                             "three_body_embedding.swish_layer.linear", False))
        real_line = bool((t_atom < n_real).any())

    def attention(key, nodes, edges, target, source, n_nodes, pair=None):
        rows = edges if pair is None else edges[pair]
        msg = _gated(torch.cat([rows, nodes[target], nodes[source]], 1), p, key + ".edge_nonlinear_update")
        att_s = _softmax_sum(_lin(rows, p, key + ".source_weight_linear", False), msg, source, n_nodes)
        att_t = _softmax_sum(_lin(rows, p, key + ".target_weight_linear", False), msg, target, n_nodes)
        new_nodes = (_gated(torch.cat([nodes, att_t, att_s], 1), p, key + ".node_nonlinear_update")
                     + nodes * p[key + ".node_res_weight"])
        m = msg if pair is None else _pair_average(msg, pair, n_u)
        return new_nodes, m + edges * p[key + ".edge_res_weight"]

    def ffn(x_, key):
        return _lin(torch.nn.functional.silu(_lin(x_, p, key + ".layers.0", False)), p, key + ".layers.3", False)

    for b in range(C.num_layers):
        pre = f"interaction_block.{b}"
        bond_in = bond
        if has_triplets:
            new_bond, trip = attention(pre + ".attn_block_line_graph", bond, trip, t_u1, t_u2, n_u)
            bond = new_bond if real_line else bond_in
        node, bond_att = attention(pre + ".attn_block_atom_graph", node, bond, centre, neighbour, n, pair=d2u)
        # without triplets the atom attention's bond update is dead: the refinement reads the block input
        bond = bond_att if has_triplets else bond_in
        if has_triplets:
            key = pre + ".refine_block_line_graph"
            env = _lin(rbf_line, p, key + ".learnable_envelope", False)
            weight = env[t_u2] * env[t_u1]
            raw = _gated(torch.cat([trip, node[t_atom], bond[t_u1], bond[t_u2]], 1), p,
                         key + ".edge_nonlinear_update")
            refined = ffn(_segment_sum(raw * weight, t_u1, n_u), key + ".node_FFN") + bond * p[key + ".node_res_weight"]
            trip = ffn(raw, key + ".edge_FFN") + trip * p[key + ".edge_res_weight"]
            bond = refined if real_line else bond_in
        key = pre + ".refine_block_atom_graph"
        rows = bond[d2u]
        weight = _lin(rbf_atom[d2u], p, key + ".learnable_envelope", False)
        raw = _gated(torch.cat([rows, node[centre], node[neighbour]], 1), p, key + ".edge_nonlinear_update")
        node_new = ffn(_segment_sum(raw * weight, centre, n), key + ".node_FFN") + node * p[key + ".node_res_weight"]
        bond = _pair_average(ffn(raw, key + ".edge_FFN"), d2u, n_u) + bond * p[key + ".edge_res_weight"]
        node = node_new

    readout = _ln(node, p, "readout_norm")
    per_atom = _mlp(readout, p, "energy_head.energy_head", len(C.energy_hidden) + 1).reshape(-1)
    energy = per_atom[:n_real].sum()
    gx, gs = torch.autograd.grad(energy, [x0, strain])
    volume = float(torch.det(lat0.detach()).abs())
    return (float(energy.detach()), (-gx).detach().numpy().astype(np.float64),
            (gs / volume * GPA).detach().numpy().astype(np.float64))
