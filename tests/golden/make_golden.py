"""Generate the golden fixtures of tests/golden/*.npz from the reference's own code.

Run in a container that holds the FastMD reference source tree (read-only):

    python tests/golden/make_golden.py /path/to/fastmd-reference [fixture ...]

It imports the reference with two stand-in modules for packages absent here
(``ase.units`` with ASE's CODATA-2014 unit definitions; nothing else of ASE is
used) and runs, on CPU:

* the reference's Triton kernels under ``TRITON_INTERPRET=1``:
  ``_aligned_gather_cat3_fwd/_bwd`` and ``_aligned_gather_cat4_fwd/_bwd``
  (fastmd/models/matris/op/triton_gather_cat.py:30/:59/:203/:236),
  ``_csr_segsum_fwd`` and ``_csr_segsum_bwd_rows``
  (fastmd/models/matris/op/triton_csr_segment_sum.py:71/:184), the segment
  attention kernels ``_csr_segment_attention_fwd/_bwd``, ``_paired_csr_segment_attention_fwd``
  and ``_paired_segment_attention_bwd_rows``
  (fastmd/models/matris/op/triton_segment_attention.py:62/:128/:210/:319), the
  decomposed indexed-concat SiLU epilogues ``_cat3/_cat4_gather_add_silu_fwd/_bwd``
  (fastmd/engine/kernels/decomposed_indexed_cat_silu_linear.py:97/:156/:234/:383), the
  MatRIS reverse-edge pairing and ordered triplets ``_build_d2u`` / ``_build_line_graph``
  (fastmd/graph/gpu_graph_builder.py:217/:511, their torch path on CPU), the
  gated-LN epilogue ``_gated_ln_fwd_2d`` / ``_gated_ln_bwd_2d``
  (fastmd/models/matris/op/triton_gated_ln.py:205/:280), the directed-pair average and
  undirected-pair expansion ``_directed_pair_average_fwd/_bwd`` / ``_undirected_pair_expand_fwd/_bwd``
  (fastmd/models/matris/op/triton_directed_pair_aggregate.py:61/:83/:105/:127), the
  residual add ``_residual_add_fwd`` / ``_residual_add_bwd``
  (fastmd/models/matris/op/triton_residual_add.py:40/:64), the float64 build prologue
  ``_float64_prologue_kernel`` (fastmd/graph/fixed_capacity_builder.py:464), the fixed-capacity
  MatRIS bond graph (the builder's ``_materialize_pairs`` / ``_materialize_line_graph`` /
  ``_substitute_overflow_topology``, :2001/:2101/:2163, called unbound on a stand-in), and the
  fixed-capacity re-filter ``_count_neighbors_kernel`` /
  ``_materialize_neighbors_kernel`` (fastmd/graph/fixed_capacity_builder.py:98/:189)
  on candidate lists of a dense search, followed by the reference's
  canonical sort key (fixed_capacity_builder.py:1978-1996);
* the radial basis ``BesselExpansion`` + ``PolynomialEnvelope``
  (fastmd/models/matris/basis_function.py:139, :31) at the MACE and MatRIS settings;
* the bundled MatRIS-10M model itself (fastmd/models/matris/model.py:99) with seeded weights, its
  energies, forces and stress in float32 and float64 on the config-0 perovskite over the reference's
  legacy CPU graph (``matris_cases``; pymatgen placeholders, the graph fed by a dense search);
* the line-graph envelope product ``_line_envelope_fwd/_bwd``
  (fastmd/models/matris/op/triton_line_envelope.py:50/:87) under the interpreter;
* the 3xTF32 wide GEMM ``_split_kernel`` + ``_wide_gemm_persistent`` / ``_wide_gemm_tiles``
  (fastmd/engine/kernels/triton_wide_gemm.py:132/:103/:120) under the interpreter, its one inline
  PTX instruction (``cvt.rna.tf32.f32``) replaced by that instruction's definition in bit operations;
* the torch backend of ``GPUNoseHooverChainNVT`` (fastmd/execution/gpu_nhc.py:709,
  ``backend="torch"``) with harmonic forces, and ``maxwell_boltzmann_momenta``
  (gpu_nhc.py:199).

The fixtures are small (a few hundred KB in total) and are the pins of the
oracle and of the GPU parity tests; nothing at test time reads the reference.
"""
from __future__ import annotations

import math
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _install_stubs() -> None:
    ase = types.ModuleType("ase")
    units = types.ModuleType("ase.units")
    _e, _amu, _k = 1.6021766208e-19, 1.660539040e-27, 1.38064852e-23  # CODATA 2014
    units.kB = _k / _e
    units.second = 1e10 * math.sqrt(_e / _amu)
    units.fs = 1e-15 * units.second
    units.Pascal = (1 / _e) / 1e30
    units.GPa = 1e9 * units.Pascal
    ase.units = units
    sys.modules["ase"] = ase
    sys.modules["ase.units"] = units


def _install_model_stubs() -> None:
    """Placeholders for the two pymatgen modules the MatRIS model module imports at load time
    (fastmd/models/matris/converter.py:9-10); the fixtures build the model's graph without them."""
    for name in ("pymatgen", "pymatgen.core", "pymatgen.io", "pymatgen.io.ase"):
        sys.modules.setdefault(name, types.ModuleType(name))
    sys.modules["pymatgen.core"].Structure = type("Structure", (), {})
    sys.modules["pymatgen.io.ase"].AseAtomsAdaptor = type("AseAtomsAdaptor", (), {})


def matris_cases(torch):
    """The reference's MatRIS-10M (fastmd/models/matris/model.py:99, ``OAM_10M`` of
    fastmd/engine/memory_admission.py:228 with energy-head widths (256, 256)) with the seeded weights of
    ``fastmd_b200.matris_params.seeded_parameters(seed=0)`` loaded into it, evaluated by ``forward(task="efs")``
    (ForceStressHead autograd forces and strain stress, readout.py:200-230) in float32 and in float64, on the
    config-0 perovskite (jitter seeds 0 and 1) over the reference's own CPU graph code (the legacy ``Graph``,
    fastmd/models/matris/legacy_graph.py:135-334, as ``GraphConverter`` builds it, converter.py:110-154) fed
    by a dense FP64 search within the 6 A cutoff in place of pymatgen's ``get_neighbor_list``."""
    _install_model_stubs()
    sys.path.insert(0, str(HERE.parents[1]))
    from fastmd.graph.geometry import small_matmul
    from fastmd.graph.radiusgraph import RadiusGraph
    from fastmd.models.matris.converter import GraphConverter
    from fastmd.models.matris.model import MatRIS
    from fastmd_b200.matris_params import MATRIS_10M, parameter_shapes, seeded_parameters
    from fastmd_b200.structures import perovskite
    from oracle.neighbors import dense_pairs

    params = seeded_parameters(MATRIS_10M, seed=0)
    model = MatRIS(**MATRIS_10M.reference_kwargs())
    state = model.state_dict()
    assert set(state) == set(params) and all(tuple(state[k].shape) == s for k, s, _ in parameter_shapes(MATRIS_10M))
    model.load_state_dict({k: torch.from_numpy(v) for k, v in params.items()})
    model.eval()
    out = {"matris_param_sum": np.array(sum(float(v.astype(np.float64).sum()) for v in params.values()))}
    for seed in (0, 1):
        pos, cell, numbers, _ = perovskite(seed=seed)
        lattice = torch.tensor(cell, dtype=torch.float32)
        frac = torch.tensor(pos @ np.linalg.inv(cell), dtype=torch.float32)
        cart = small_matmul(frac, lattice)  # the coordinates the model sees (processgraph.py:96)
        pairs = dense_pairs(cart.double().numpy(), cell, MATRIS_10M.pairwise_cutoff)
        keys = sorted(pairs)
        graph = GraphConverter._create_graph_legacy(
            len(numbers), np.array([k[0] for k in keys]), np.array([k[1] for k in keys]),
            np.array([k[2:] for k in keys], dtype=np.float64), np.array([pairs[k] for k in keys]))
        atom_graph, d2u = graph.adjacency_list()
        u2d = graph.undirected2directed()
        line = graph.line_graph_adjacency_list(cutoff=MATRIS_10M.three_body_cutoff)
        images = np.array([e.info["image"] for e in graph.directed_edges_list], dtype=np.float64)
        tag = f"matris_s{seed}"
        # the float64 evaluation's own coordinates (frac @ L in float64 of the same float32 inputs)
        out[f"{tag}_positions64"] = small_matmul(frac.double(), lattice.double()).numpy()
        out.update({f"{tag}_positions": cart.numpy(), f"{tag}_cell": lattice.numpy(), f"{tag}_numbers": numbers,
                    f"{tag}_edge_index": np.asarray(atom_graph, np.int32).reshape(-1, 2),
                    f"{tag}_edge_image": images.astype(np.float32), f"{tag}_d2u": np.asarray(d2u, np.int32),
                    f"{tag}_u2d": np.asarray(u2d, np.int32), f"{tag}_line_graph": np.asarray(line, np.int32).reshape(-1, 5)})
        for dtype, name in ((torch.float32, "32"), (torch.float64, "64")):
            radius_graph = RadiusGraph(
                graph_id=None, mp_id=None, composition=None, atomic_number=torch.tensor(numbers, dtype=torch.int32),
                atom_frac_coord=frac.to(dtype), lattice=lattice.to(dtype),
                neighbor_image=torch.tensor(images, dtype=dtype), atom_graph=torch.tensor(out[f"{tag}_edge_index"]),
                atom_graph_cutoff=MATRIS_10M.pairwise_cutoff, line_graph=torch.tensor(out[f"{tag}_line_graph"]),
                line_graph_cutoff=MATRIS_10M.three_body_cutoff, directed2undirected=torch.tensor(out[f"{tag}_d2u"]),
                undirected2directed=torch.tensor(out[f"{tag}_u2d"]))
            pred = model.to(dtype)([radius_graph], task="efs")
            # "e" is per atom (is_intensive); the extensive energy is e * n (the adapter's extensive_energy)
            out[f"{tag}_e{name}"] = np.array(float(pred["e"].double().item()) * len(numbers))
            out[f"{tag}_f{name}"] = pred["f"][0].detach().double().numpy()
            out[f"{tag}_s{name}"] = pred["s"][0].detach().double().numpy()
        model.float()
    return out


def line_envelope_cases(torch, le):
    """The reference's line-graph envelope product and its backward, ``_line_envelope_fwd`` /
    ``_line_envelope_bwd`` (fastmd/models/matris/op/triton_line_envelope.py:50/:87), under the interpreter,
    on a random bond table and triplet index pairs (source = column 3, target = column 1 of a line graph)."""
    rng = np.random.default_rng(21)
    out = {}
    for tag, (U, T, D) in {"small": (37, 301, 32), "wide": (40, 256, 128)}.items():
        base = rng.standard_normal((U, D)).astype(np.float32)
        target = rng.integers(0, U, T).astype(np.int64)
        source = rng.integers(0, U, T).astype(np.int64)
        gout = rng.standard_normal((T, D)).astype(np.float32)
        tb, ts, tt, tg = (torch.from_numpy(x) for x in (base, source, target, gout))
        env = torch.empty((T, D))
        BM, BD = 16, min(D, 128)
        grid = ((T + BM - 1) // BM, (D + BD - 1) // BD)
        le._line_envelope_fwd[grid](tb, ts, tt, env, T, D=D, S0=D, BM=BM, BD=BD)
        grad = torch.zeros((U, D))
        le._line_envelope_bwd[grid](tg, tb, ts, tt, grad, T, D=D, S0=D, GS0=D, BM=BM, BD=BD)
        out.update({f"env_{tag}_base": base, f"env_{tag}_source": source, f"env_{tag}_target": target,
                    f"env_{tag}_gout": gout, f"env_{tag}_out": env.numpy(), f"env_{tag}_grad": grad.numpy()})
    return out


def wide_gemm_cases(torch, wg):
    """The reference's 3xTF32 wide GEMM (fastmd/engine/kernels/triton_wide_gemm.py): ``_split_kernel`` (:132)
    for the K-major weight pairs, then ``_wide_gemm_persistent`` (:103, K <= 256) or ``_wide_gemm_tiles`` (:120,
    K >= 384) on tensor descriptors, with the launch geometry of ``_launch`` (:297: 128-row tiles, BN = min(128, N),
    BK 64), under the interpreter. The interpreter cannot execute the kernel's one inline PTX instruction
    (``cvt.rna.tf32.f32`` in ``_rna_tf32``, :63), so that function is replaced by the instruction's definition in
    bit operations (round to nearest, ties away from zero, the low 13 bits cleared); everything else is the
    reference's code. The interpreter's dots are FP32 products of the given operands (the TF32 parts exact), so
    these outputs are the reference's algorithm (term set and order, 64-wide chunks on fresh accumulators summed in
    FP32, bias then c) at FP32 rounding."""
    import triton
    from triton.tools.tensor_descriptor import TensorDescriptor

    from _rna_tf32_definition import rna_tf32 as _rna_tf32_definition
    from inputs import WIDE_GEMM_CASES, wide_gemm_inputs

    wg._rna_tf32 = _rna_tf32_definition
    out = {}
    # the inputs are counter streams (tests/golden/inputs.py), regenerated by the tests: only outputs are stored
    for i, (tag, (m, k, n, transposed, has_bias, has_c)) in enumerate(WIDE_GEMM_CASES.items()):
        a, w, bias, c = wide_gemm_inputs(i, m, k, n, transposed, has_bias, has_c)
        tw = torch.from_numpy(w)
        src = tw.t() if transposed else tw  # the K-major [N, K] operand
        hi = torch.empty(src.shape)
        lo = torch.empty(src.shape)
        total = n * k
        wg._split_kernel[(triton.cdiv(total, 1024),)](src, hi, lo, total, COLS=k, S_ROW=src.stride(0),
                                                       S_COL=src.stride(1), BLOCK=1024)
        ta = torch.from_numpy(a)
        y = torch.empty((m, n))
        bm, bn = 128, min(128, n)
        args = (TensorDescriptor.from_tensor(ta, [bm, wg._BK]), TensorDescriptor.from_tensor(hi, [bn, wg._BK]),
                TensorDescriptor.from_tensor(lo, [bn, wg._BK]), torch.from_numpy(c) if has_c else y,
                TensorDescriptor.from_tensor(y, [bm, bn]), torch.from_numpy(bias) if has_bias else hi, m)
        consts = dict(K=k, NT_N=n // bn, BM=bm, BN=bn, BK=wg._BK, PREC="tf32x3", HAS_BIAS=has_bias, HAS_C=has_c)
        tiles = triton.cdiv(m, bm) * (n // bn)
        if k >= 384:
            wg._wide_gemm_tiles[(tiles,)](*args, **consts)
        else:  # persistent programs: min(tiles, SMs) of a 148-SM device
            wg._wide_gemm_persistent[(min(tiles, 148),)](*args, **consts)
        out[f"wg_{tag}_y"] = y.numpy()
        out[f"wg_{tag}_shape"] = np.array([m, k, n, transposed, has_bias, has_c], dtype=np.int64)
        if tag == "k64_n64_bias":  # the reference's K-major split of one weight, for the bitwise split check
            out[f"wg_{tag}_hi"] = hi.numpy()
            out[f"wg_{tag}_lo"] = lo.numpy()
    return out


def gather_cat_cases(torch, gc):
    out = {}
    rng = np.random.default_rng(11)
    for tag, (E, N, D) in {"small": (37, 11, 8), "wide": (53, 17, 128), "odd": (29, 7, 5)}.items():
        A = rng.standard_normal((E, D)).astype(np.float32)
        X = rng.standard_normal((N, D)).astype(np.float32)
        ia = np.sort(rng.integers(0, N, E)).astype(np.int64)  # sorted (receiver-like)
        ib = rng.integers(0, N, E).astype(np.int64)            # unsorted (sender-like)
        G = rng.standard_normal((E, 3 * D)).astype(np.float32)
        block = 1 << (D - 1).bit_length()
        t = {k: torch.from_numpy(v) for k, v in dict(A=A, X=X, ia=ia, ib=ib, G=G).items()}
        y = torch.empty(E, 3 * D)
        gc._aligned_gather_cat3_fwd[(E,)](t["A"], t["X"], t["ia"], t["ib"], y, E, D=D, BLK=block,
                                          S0_STRIDE=D, S1_STRIDE=D)
        ga = torch.empty(E, D)
        gx = torch.zeros(N, D)
        gc._aligned_gather_cat3_bwd[(E,)](ga, gx, t["ia"], t["ib"], t["G"], E, D=D, BLK=block)
        out.update({f"cat3_{tag}_{k}": v for k, v in dict(A=A, X=X, ia=ia, ib=ib, G=G).items()})
        out[f"cat3_{tag}_out"] = y.numpy()
        out[f"cat3_{tag}_grad_aligned"] = ga.numpy()
        out[f"cat3_{tag}_grad_gathered"] = gx.numpy()
    # cat4: [A | Xa[ia] | Xb[ib] | Xb[ic]]
    E, Na, Nb, D = 41, 9, 13, 16
    A = rng.standard_normal((E, D)).astype(np.float32)
    Xa = rng.standard_normal((Na, D)).astype(np.float32)
    Xb = rng.standard_normal((Nb, D)).astype(np.float32)
    ia = rng.integers(0, Na, E).astype(np.int64)
    ib = rng.integers(0, Nb, E).astype(np.int64)
    ic = rng.integers(0, Nb, E).astype(np.int64)
    G = rng.standard_normal((E, 4 * D)).astype(np.float32)
    t = {k: torch.from_numpy(v) for k, v in dict(A=A, Xa=Xa, Xb=Xb, ia=ia, ib=ib, ic=ic, G=G).items()}
    y = torch.empty(E, 4 * D)
    gc._aligned_gather_cat4_fwd[(E,)](t["A"], t["Xa"], t["ia"], t["Xb"], t["ib"], t["ic"], y, E, D=D, BLK=D,
                                      S0_STRIDE=D, S1_STRIDE=D, S2_STRIDE=D)
    g0, g1, g2 = torch.empty(E, D), torch.zeros(Na, D), torch.zeros(Nb, D)
    gc._aligned_gather_cat4_bwd[(E,)](g0, g1, g2, t["ia"], t["ib"], t["ic"], t["G"], E, D=D, BLK=D)
    out.update({f"cat4_{k}": v for k, v in dict(A=A, Xa=Xa, Xb=Xb, ia=ia, ib=ib, ic=ic, G=G).items()})
    out.update(cat4_out=y.numpy(), cat4_grad_aligned=g0.numpy(), cat4_grad_a=g1.numpy(), cat4_grad_b=g2.numpy())
    return out


def segment_sum_cases(torch, cs):
    out = {}
    rng = np.random.default_rng(12)
    cases = {"identity": (200, 23, 32, True, False, -1), "perm_weighted": (301, 37, 20, False, True, -1),
             "wide_skip": (150, 11, 128, True, True, 4), "narrow": (97, 13, 3, False, False, -1)}
    for tag, (rows, S, D, identity, weighted, skip) in cases.items():
        seg = rng.integers(0, S, rows).astype(np.int64)
        if identity:
            seg = np.sort(seg)
        perm = np.argsort(seg, kind="stable").astype(np.int64)
        off = np.searchsorted(seg[perm], np.arange(S + 1)).astype(np.int64)
        V = rng.standard_normal((rows, D)).astype(np.float32)
        W = rng.standard_normal((rows, D)).astype(np.float32)
        G = rng.standard_normal((S, D)).astype(np.float32)
        t = {k: torch.from_numpy(v) for k, v in dict(seg=seg, perm=perm, off=off, V=V, W=W, G=G).items()}
        y = torch.empty(S, D)
        bd = min(1 << (D - 1).bit_length(), 128)
        cs._csr_segsum_fwd[(S, (D + bd - 1) // bd)](
            t["V"], t["W"] if weighted else t["V"], t["off"] if identity else t["perm"], t["off"], y, S, skip,
            D=D, VAL_S0=D, VAL_S1=1, W_S0=D, W_S1=1, BS=1, BR=16, BD=bd, IDENTITY_PERM=identity,
            WEIGHTED=weighted, HAS_SKIP=skip >= 0, ACC_FP64=False)
        gv, gw = torch.empty(rows, D), torch.empty(rows, D)
        cs._csr_segsum_bwd_rows[((rows + 31) // 32, (D + bd - 1) // bd)](
            t["G"], t["V"], t["W"] if weighted else t["V"], t["seg"], gv, gw, rows, skip, D=D, SEG_S0=1,
            VAL_S0=D, VAL_S1=1, W_S0=D, W_S1=1, BM=32, BD=bd, WEIGHTED=weighted, NEED_GV=True,
            NEED_GW=weighted, HAS_SKIP=skip >= 0)
        out.update({f"segsum_{tag}_{k}": v for k, v in dict(seg=seg, perm=perm, off=off, V=V, W=W, G=G).items()})
        out[f"segsum_{tag}_meta"] = np.array([S, int(identity), int(weighted), skip], dtype=np.int64)
        out[f"segsum_{tag}_out"] = y.numpy()
        out[f"segsum_{tag}_gvalue"] = gv.numpy()
        if weighted:
            out[f"segsum_{tag}_gweight"] = gw.numpy()
    return out


def segment_attention_cases(torch, sa):
    """``_csr_segment_attention_fwd/_bwd`` and the paired forward / row backward
    (fastmd/models/matris/op/triton_segment_attention.py:62/:128/:210/:319)."""
    out = {}
    rng = np.random.default_rng(13)
    # rows, segments, width, identity CSR, skip segment, lse
    cases = {"perm_lse": (120, 17, 32, False, -1, True), "identity_skip": (90, 12, 128, True, 11, False),
             "odd_lse_skip": (77, 9, 5, False, 3, True), "wide_empty": (64, 40, 64, False, -1, True)}
    for tag, (rows, S, D, identity, skip, lse) in cases.items():
        seg = rng.integers(0, S, rows).astype(np.int64)
        if tag == "wide_empty":
            seg = rng.choice(np.arange(0, S, 3), rows).astype(np.int64)  # two thirds of the segments empty
        if identity:
            seg = np.sort(seg)
        perm = np.argsort(seg, kind="stable").astype(np.int64)
        off = np.searchsorted(seg[perm], np.arange(S + 1)).astype(np.int64)
        L = (3.0 * rng.standard_normal((rows, D))).astype(np.float32)
        V = rng.standard_normal((rows, D)).astype(np.float32)
        G = rng.standard_normal((S, D)).astype(np.float32)
        GL = rng.standard_normal((S, D)).astype(np.float32)
        t = {k: torch.from_numpy(v) for k, v in dict(seg=seg, perm=perm, off=off, L=L, V=V, G=G, GL=GL).items()}
        blk = 1 << (D - 1).bit_length()
        y = torch.empty(S, D)
        ls = torch.empty(S, D) if lse else None
        sa._csr_segment_attention_fwd[(S,)](
            t["L"], t["V"], t["seg"] if identity else t["perm"], t["off"], y, ls, skip, D=D, LOG_S0=D, LOG_S1=1,
            VAL_S0=D, VAL_S1=1, BLK=blk, IDENTITY_PERM=identity, HAS_SKIP=skip >= 0, STORE_LSE=lse)
        gl = torch.zeros(rows, D)
        gv = torch.zeros(rows, D)
        sa._csr_segment_attention_bwd[(S,)](
            t["L"], t["V"], y, t["G"], t["seg"] if identity else t["perm"], t["off"], gl, gv,
            t["GL"] if lse else None, skip, D=D, LOG_S0=D, LOG_S1=1, VAL_S0=D, VAL_S1=1, GL_S0=D, BLK=blk,
            IDENTITY_PERM=identity, HAS_SKIP=skip >= 0, HAS_GLSE=lse)
        out.update({f"sa_{tag}_{k}": v for k, v in dict(seg=seg, perm=perm, off=off, L=L, V=V, G=G).items()})
        if lse:
            out[f"sa_{tag}_GL"] = GL
            out[f"sa_{tag}_lse"] = ls.numpy()
        out[f"sa_{tag}_meta"] = np.array([S, int(identity), skip, int(lse)], dtype=np.int64)
        out[f"sa_{tag}_out"] = y.numpy()
        out[f"sa_{tag}_glogits"] = gl.numpy()
        out[f"sa_{tag}_gvalue"] = gv.numpy()
    # paired: two CSRs over the same rows sharing the values
    for tag, (rows, S, D, skip, lse) in {"pair": (110, 14, 32, -1, True), "pair_skip": (96, 10, 20, 9, False)}.items():
        sa_, sb_ = rng.integers(0, S, rows).astype(np.int64), rng.integers(0, S, rows).astype(np.int64)
        pa, pb = np.argsort(sa_, kind="stable").astype(np.int64), np.argsort(sb_, kind="stable").astype(np.int64)
        oa = np.searchsorted(sa_[pa], np.arange(S + 1)).astype(np.int64)
        ob = np.searchsorted(sb_[pb], np.arange(S + 1)).astype(np.int64)
        La = (2.0 * rng.standard_normal((rows, D))).astype(np.float32)
        Lb = (2.0 * rng.standard_normal((rows, D))).astype(np.float32)
        V = rng.standard_normal((rows, D)).astype(np.float32)
        Ga, Gb = rng.standard_normal((S, D)).astype(np.float32), rng.standard_normal((S, D)).astype(np.float32)
        GLa, GLb = rng.standard_normal((S, D)).astype(np.float32), rng.standard_normal((S, D)).astype(np.float32)
        arrays = dict(sa=sa_, sb=sb_, pa=pa, pb=pb, oa=oa, ob=ob, La=La, Lb=Lb, V=V, Ga=Ga, Gb=Gb, GLa=GLa, GLb=GLb)
        t = {k: torch.from_numpy(v) for k, v in arrays.items()}
        blk = 1 << (D - 1).bit_length()
        res = {k: torch.empty(S, D) for k in ("out_a", "out_b", "max_a", "denom_a", "max_b", "denom_b")}
        lse_a, lse_b = (torch.empty(S, D), torch.empty(S, D)) if lse else (None, None)
        sa._paired_csr_segment_attention_fwd[(S,)](
            t["La"], t["Lb"], t["V"], t["pa"], t["oa"], t["pb"], t["ob"], res["out_a"], res["out_b"], res["max_a"],
            res["denom_a"], res["max_b"], res["denom_b"], lse_a, lse_b, skip, D=D, LOGA_S0=D, LOGA_S1=1,
            LOGB_S0=D, LOGB_S1=1, VAL_S0=D, VAL_S1=1, BLK=blk, IDENTITY_A=False, IDENTITY_B=False,
            HAS_SKIP=skip >= 0, STORE_LSE=lse)
        gla, glb, gv = torch.empty(rows, D), torch.empty(rows, D), torch.empty(rows, D)
        bd = min(blk, 128)
        sa._paired_segment_attention_bwd_rows[((rows + 7) // 8, (D + bd - 1) // bd)](
            t["La"], t["Lb"], t["V"], t["Ga"], t["Gb"], res["out_a"], res["out_b"], res["max_a"], res["denom_a"],
            res["max_b"], res["denom_b"], t["sa"], t["sb"], gla, glb, gv, t["GLa"] if lse else None,
            t["GLb"] if lse else None, rows, skip, D=D, LOGA_S0=D, LOGA_S1=1, LOGB_S0=D, LOGB_S1=1, VAL_S0=D,
            VAL_S1=1, GLA_S0=D, GLB_S0=D, BM=8, BD=bd, HAS_SKIP=skip >= 0, HAS_GLSE=lse)
        out.update({f"psa_{tag}_{k}": v for k, v in arrays.items()})
        out[f"psa_{tag}_meta"] = np.array([S, skip, int(lse)], dtype=np.int64)
        out.update({f"psa_{tag}_{k}": v.numpy() for k, v in res.items()})
        if lse:
            out[f"psa_{tag}_lse_a"], out[f"psa_{tag}_lse_b"] = lse_a.numpy(), lse_b.numpy()
        out[f"psa_{tag}_glogits_a"], out[f"psa_{tag}_glogits_b"] = gla.numpy(), glb.numpy()
        out[f"psa_{tag}_gvalue"] = gv.numpy()
    return out


def gather_add_silu_cases(torch, di):
    """The decomposed indexed-concat epilogues ``_cat3_gather_add_silu_fwd/_bwd`` and
    ``_cat4_gather_add_silu_fwd/_bwd`` (fastmd/engine/kernels/decomposed_indexed_cat_silu_linear.py:97,
    :156, :234, :383): preact = p0 + p1[ia] + p2[ib] (+ p3[ic]) + bias, SiLU of its core / gate halves,
    and the backward's SiLU derivative with its scatter into the gathered projections."""
    out = {}
    rng = np.random.default_rng(14)
    for tag, (M, NS, H, cat4, sorted_a, bias) in {"cat3": (57, 13, 16, False, False, True),
                                                  "cat3_sorted_odd": (45, 9, 12, False, True, False),
                                                  "cat4": (38, 11, 8, True, False, True)}.items():
        N = 2 * H
        blk = 1 << (H - 1).bit_length()
        ia = rng.integers(0, NS, M).astype(np.int64)
        if sorted_a:
            ia = np.sort(ia)
        ib = rng.integers(0, NS, M).astype(np.int64)
        ic = rng.integers(0, NS, M).astype(np.int64)
        arr = dict(p0=rng.standard_normal((M, N)), p1=rng.standard_normal((NS, N)), p2=rng.standard_normal((NS, N)),
                   p3=rng.standard_normal((NS, N)), b=rng.standard_normal(N), gc=rng.standard_normal((M, H)),
                   gg=rng.standard_normal((M, H)))
        arr = {k: (2.0 * v).astype(np.float32) for k, v in arr.items()}
        arr.update(ia=ia, ib=ib, ic=ic)
        t = {k: torch.from_numpy(v) for k, v in arr.items()}
        pre, ca, ga = torch.empty(M, N), torch.empty(M, H), torch.empty(M, H)
        gp = [torch.zeros(M, N)] + [torch.zeros(NS, N) for _ in range(3)]
        bias_t = t["b"] if bias else None
        if cat4:
            di._cat4_gather_add_silu_fwd[((M + 7) // 8,)](
                t["p0"], t["p1"], t["p2"], t["p3"], t["ia"], t["ib"], t["ic"], bias_t, pre, ca, ga, SIA=1, SIB=1,
                SIC=1, SP0=N, M=M, H=H, N=N, BM=8, BLK=blk, HAS_BIAS=bias)
            di._cat4_gather_add_silu_bwd[((M + 7) // 8,)](
                t["gc"], t["gg"], pre, t["ia"], t["ib"], t["ic"], gp[0], gp[1], gp[2], gp[3], SIA=1, SIB=1, SIC=1,
                M=M, H=H, N=N, BM=8, BLK=blk, SORTED_A=sorted_a)
        else:
            di._cat3_gather_add_silu_fwd[((M + 7) // 8,)](
                t["p0"], t["p1"], t["p2"], t["ia"], t["ib"], bias_t, pre, ca, ga, SIA=1, SIB=1, SP0=N, M=M, H=H,
                N=N, BM=8, BLK=blk, HAS_BIAS=bias)
            di._cat3_gather_add_silu_bwd[((M + 7) // 8,)](
                t["gc"], t["gg"], pre, t["ia"], t["ib"], gp[0], gp[1], gp[2], SIA=1, SIB=1, M=M, H=H, N=N, BM=8,
                BLK=blk, SORTED_A=sorted_a)
        out.update({f"gas_{tag}_{k}": v for k, v in arr.items()})
        out[f"gas_{tag}_meta"] = np.array([M, NS, H, int(cat4), int(sorted_a), int(bias)], dtype=np.int64)
        out[f"gas_{tag}_preact"], out[f"gas_{tag}_core"], out[f"gas_{tag}_gate"] = pre.numpy(), ca.numpy(), ga.numpy()
        for k in range(4 if cat4 else 3):
            out[f"gas_{tag}_gp{k}"] = gp[k].numpy()
    return out


def pairs_line_graph_cases(torch, ggb):
    """MatRIS reverse-edge pairing ``_build_d2u`` and the ordered triplets ``_build_line_graph``
    (fastmd/graph/gpu_graph_builder.py:217, :511) on dense FP64 neighbour lists of a perovskite
    (canonically sorted edges), a small triclinic cell with many images (edges shuffled) and a
    sparse box with isolated atoms."""
    sys.path.insert(0, str(HERE.parents[1]))
    from oracle.neighbors import dense_pairs

    out = {}
    rng = np.random.default_rng(15)
    a = 6.2
    basis = np.array([[0, 0, 0], [.5, .5, .5], [.5, .5, 0], [.5, 0, .5], [0, .5, .5]])
    grid = np.array([[i, j, k] for i in range(3) for j in range(3) for k in range(3)], float)
    perov = ((grid[:, None] + basis[None]).reshape(-1, 3) * a + rng.normal(0, 0.05, (135, 3)), np.eye(3) * 3 * a)
    tric_cell = np.array([[4.0, 0.0, 0.0], [1.1, 3.8, 0.0], [0.7, 0.9, 4.2]])
    tric = (rng.uniform(0, 1, (6, 3)) @ tric_cell, tric_cell)
    sparse = (np.concatenate([rng.uniform(0, 3, (4, 3)), rng.uniform(10, 20, (5, 3))]), np.eye(3) * 30.0)
    for tag, ((pos, cell), rc, line_cut, presorted) in {"perov": (perov, 6.0, 4.5, True),
                                                        "triclinic": (tric, 5.0, 3.2, False),
                                                        "sparse": (sparse, 4.0, 2.5, False)}.items():
        pairs = dense_pairs(pos, cell, rc)
        keys = sorted(pairs)
        center = np.array([k[0] for k in keys], np.int64)
        neighbor = np.array([k[1] for k in keys], np.int64)
        images = np.array([k[2:] for k in keys], np.int32).reshape(-1, 3)
        dist = np.array([pairs[k] for k in keys], np.float32)
        if not presorted:
            order = rng.permutation(len(keys))
            center, neighbor, images, dist = center[order], neighbor[order], images[order], dist[order]
        n = pos.shape[0]
        d2u, u2d = ggb._build_d2u(torch.from_numpy(center), torch.from_numpy(neighbor),
                                  torch.from_numpy(images.astype(np.int64)), n, presorted=presorted)
        lg = ggb._build_line_graph(torch.from_numpy(center), d2u, torch.from_numpy(dist), n, line_cut,
                                   presorted=presorted)
        out.update({f"plg_{tag}_{k}": v for k, v in dict(center=center, neighbor=neighbor, images=images,
                                                             dist=dist).items()})
        out[f"plg_{tag}_meta"] = np.array([n, int(presorted)], dtype=np.int64)
        out[f"plg_{tag}_cutoff"] = np.array([line_cut], dtype=np.float32)
        out[f"plg_{tag}_d2u"], out[f"plg_{tag}_u2d"] = d2u.numpy(), u2d.numpy()
        out[f"plg_{tag}_triplets"] = lg.numpy()
    return out


def gated_ln_cases(torch, gl):
    """The fused GatedMLP epilogue ``silu(LN(core)) * sigmoid(LN(gate)) (+ res_weight * residual)``:
    the reference's default 2-D tile kernels ``_gated_ln_fwd_2d`` / ``_gated_ln_bwd_2d``
    (fastmd/models/matris/op/triton_gated_ln.py:205, :280), tiles from its ``_tile_2d``."""
    out = {}
    rng = np.random.default_rng(16)
    for tag, (rows, D, residual, bias) in {"w128_res_bias": (37, 128, True, True), "w32": (45, 32, False, False),
                                           "w24_bias": (29, 24, False, True), "w128_res": (20, 128, True, False)}.items():
        blk = 1 << (D - 1).bit_length()
        arr = dict(cx=2 * rng.standard_normal((rows, D)) + 0.5, gx=rng.standard_normal((rows, D)),
                   cw=1 + 0.3 * rng.standard_normal(D), cb=0.2 * rng.standard_normal(D),
                   gw=1 + 0.3 * rng.standard_normal(D), gb=0.2 * rng.standard_normal(D),
                   clb=0.5 * rng.standard_normal(D), glb=0.5 * rng.standard_normal(D),
                   res=rng.standard_normal((rows, D)), rw=rng.standard_normal(D), g=rng.standard_normal((rows, D)))
        arr = {k: v.astype(np.float32) for k, v in arr.items()}
        t = {k: torch.from_numpy(v) for k, v in arr.items()}
        y = torch.empty(rows, D)
        stats = [torch.empty(rows) for _ in range(4)]
        bm, _ = gl._tile_2d(blk, False)
        gl._gated_ln_fwd_2d[((rows + bm - 1) // bm,)](
            t["cx"], t["gx"], t["clb"] if bias else t["cw"], t["glb"] if bias else t["cw"], t["cw"], t["cb"], t["gw"],
            t["gb"], t["res"] if residual else t["cx"], t["rw"] if residual else t["cw"], y, *stats, rows, D=D, BLK=blk,
            BM=bm, EPS_CORE=1e-5, EPS_GATE=1e-5, HAS_RESIDUAL=residual, HAS_BIAS=bias)
        gc, gg, gr = torch.empty(rows, D), torch.empty(rows, D), torch.empty(rows, D)
        bmb, _ = gl._tile_2d(blk, True)
        gl._gated_ln_bwd_2d[((rows + bmb - 1) // bmb,)](
            t["cx"], t["gx"], t["clb"] if bias else t["cw"], t["glb"] if bias else t["cw"], t["cw"], t["cb"], t["gw"],
            t["gb"], t["rw"] if residual else t["cw"], t["g"], *stats, gc, gg, gr if residual else gc, rows, D=D,
            BLK=blk, BM=bmb, HAS_RESIDUAL=residual, HAS_BIAS=bias)
        out.update({f"gln_{tag}_{k}": v for k, v in arr.items()})
        out[f"gln_{tag}_meta"] = np.array([rows, D, int(residual), int(bias)], dtype=np.int64)
        out[f"gln_{tag}_out"] = y.numpy()
        for k, v in zip(("cmean", "crstd", "gmean", "grstd"), stats):
            out[f"gln_{tag}_{k}"] = v.numpy()
        out[f"gln_{tag}_gcore"], out[f"gln_{tag}_ggate"] = gc.numpy(), gg.numpy()
        if residual:
            out[f"gln_{tag}_gres"] = gr.numpy()
    return out


def pair_aggregate_cases(torch, pa):
    """Directed-edge <-> undirected-pair aggregation: the reference's ``_directed_pair_average_fwd/_bwd``
    and ``_undirected_pair_expand_fwd/_bwd`` (fastmd/models/matris/op/triton_directed_pair_aggregate.py:61,
    :83, :105, :127) on a shuffled pair bijection, launched as its wrappers launch them (BM 8,
    BD = next_pow2(min(128, D)), grid (cdiv(U, BM), cdiv(D, 128))); the inputs are column views of a
    wider buffer (row stride ``S0``) where the case says so."""
    out = {}
    rng = np.random.default_rng(17)
    for tag, (U, D, stride) in {"d32": (23, 32, 32), "d128_strided": (24, 128, 192), "d5": (9, 5, 5)}.items():
        seg = np.repeat(np.arange(U), 2)[rng.permutation(2 * U)]
        pair = np.argsort(seg, kind="stable").reshape(U, 2).astype(np.int64)
        base = rng.standard_normal((2 * U, stride)).astype(np.float32)
        gavg = rng.standard_normal((U, D)).astype(np.float32)
        und = rng.standard_normal((U, stride)).astype(np.float32)
        gexp = rng.standard_normal((2 * U, D)).astype(np.float32)
        bd = min(1 << (D - 1).bit_length(), 128)
        grid = ((U + 7) // 8, (D + 127) // 128)
        t_pair = torch.from_numpy(pair)
        avg, gdata = torch.empty(U, D), torch.empty(2 * U, D)
        exp, gund = torch.empty(2 * U, D), torch.empty(U, D)
        pa._directed_pair_average_fwd[grid](torch.from_numpy(base), t_pair, avg, U, D=D, S0=stride, BM=8, BD=bd)
        pa._directed_pair_average_bwd[grid](torch.from_numpy(gavg), t_pair, gdata, U, D=D, BM=8, BD=bd)
        pa._undirected_pair_expand_fwd[grid](torch.from_numpy(und), t_pair, exp, U, D=D, S0=stride, BM=8, BD=bd)
        pa._undirected_pair_expand_bwd[grid](torch.from_numpy(gexp), t_pair, gund, U, D=D, BM=8, BD=bd)
        out.update({f"pa_{tag}_base": base, f"pa_{tag}_pair": pair, f"pa_{tag}_gavg": gavg, f"pa_{tag}_und": und,
                    f"pa_{tag}_gexp": gexp, f"pa_{tag}_meta": np.array([U, D, stride], dtype=np.int64),
                    f"pa_{tag}_avg": avg.numpy(), f"pa_{tag}_gdata": gdata.numpy(), f"pa_{tag}_exp": exp.numpy(),
                    f"pa_{tag}_gund": gund.numpy()})
    return out


def residual_add_cases(torch, ra):
    """The MatRIS residual add with a frozen weight: the reference's ``_residual_add_fwd`` /
    ``_residual_add_bwd`` (fastmd/models/matris/op/triton_residual_add.py:40, :64) launched as its
    wrapper launches them (BD = next_pow2(min(128, D)), BM 8, grid (cdiv(N, BM), cdiv(D, BD))); delta,
    residual and out are column views of wider buffers (row strides ``sd``, ``sr``, ``so``) where the
    case says so; out is contiguous, as the wrapper's ``empty_like`` of a row-strided view is."""
    out = {}
    rng = np.random.default_rng(23)
    for tag, (n, d, sd, sr) in {"d128": (37, 128, 128, 128), "d64_strided": (20, 64, 96, 80),
                                "d5": (9, 5, 5, 5)}.items():
        delta = rng.standard_normal((n, sd)).astype(np.float32)
        residual = rng.standard_normal((n, sr)).astype(np.float32)
        weight = rng.standard_normal(d).astype(np.float32)
        gout = rng.standard_normal((n, d)).astype(np.float32)
        bd = min(1 << (d - 1).bit_length(), 128)
        grid = ((n + 7) // 8, (d + bd - 1) // bd)
        res = torch.empty(n, d)
        ra._residual_add_fwd[grid](torch.from_numpy(delta), torch.from_numpy(residual), torch.from_numpy(weight),
                                   res, n, d, sd, sr, d, 8, bd)
        gres = torch.empty(n, d)
        ra._residual_add_bwd[grid](torch.from_numpy(gout), torch.from_numpy(weight), gres, N=n, D=d, BM=8, BD=bd)
        out.update({f"ra_{tag}_delta": delta, f"ra_{tag}_residual": residual, f"ra_{tag}_weight": weight,
                    f"ra_{tag}_gout": gout, f"ra_{tag}_meta": np.array([n, d, sd, sr], dtype=np.int64),
                    f"ra_{tag}_out": res.numpy(), f"ra_{tag}_gres": gres.numpy()})
    return out


def nhc_cases(torch, gpu_nhc):
    from ase import units

    out = {}
    rng = np.random.default_rng(13)
    n = 10
    masses = rng.uniform(1.0, 140.0, n)
    q0 = rng.uniform(0.0, 8.0, (n, 3))
    k_spring = 1.7

    def harmonic(q, dtype):
        f = -k_spring * (q - q0)
        e = 0.5 * k_spring * float(np.sum((q - q0) ** 2))
        return f.astype(dtype), e

    cases = {"f64_m3_l1": (3, 1, np.float64), "f32_m3_l1": (3, 1, np.float32), "f64_m1_l1": (1, 1, np.float64),
             "f64_m5_l2": (5, 2, np.float64)}
    steps = 60
    for tag, (tchain, tloop, fdtype) in cases.items():
        momenta = gpu_nhc.maxwell_boltzmann_momenta(masses, 300.0, seed=0)
        q_start = q0 + rng.normal(0.0, 0.1, (n, 3))
        nhc = gpu_nhc.GPUNoseHooverChainNVT(
            masses, q_start, momenta, temperature_K=300.0, timestep=1.0 * units.fs, tdamp=100.0 * units.fs,
            tchain=tchain, tloop=tloop, device="cpu", backend="torch",
            force_dtype=torch.float32 if fdtype == np.float32 else torch.float64)
        f, e = harmonic(q_start, fdtype)
        nhc.set_forces(torch.from_numpy(f), energy=torch.tensor([e], dtype=torch.float64))
        flats = [nhc.state.flat.numpy().copy()]
        for _ in range(steps):
            q = nhc.step_pre_force().numpy().copy()
            f, e = harmonic(q, fdtype)
            nhc.step_post_force(torch.from_numpy(f), energy=torch.tensor([e], dtype=torch.float64))
            flats.append(nhc.state.flat.numpy().copy())
        out[f"nhc_{tag}_flat"] = np.array(flats)
        out[f"nhc_{tag}_init"] = np.concatenate([masses, q_start.ravel(), momenta.ravel()])
        out[f"nhc_{tag}_meta"] = np.array([n, tchain, tloop, int(fdtype == np.float32), steps], dtype=np.int64)
    out["nhc_params"] = np.array([300.0, 1.0 * units.fs, 100.0 * units.fs, k_spring], dtype=np.float64)
    out["nhc_q0"] = q0
    # Maxwell-Boltzmann momenta of the 135-atom ABX3 masses at 500 K, seed 0
    perov_masses = np.array([132.905, 118.71, 126.904, 126.904, 126.904] * 27)
    out["mb_masses"] = perov_masses
    out["mb_momenta_500K_seed0"] = gpu_nhc.maxwell_boltzmann_momenta(perov_masses, 500.0, seed=0)
    return out


def neighbor_cases(torch, fcb):
    """The reference's fixed-capacity re-filter on dense candidate lists (wrapped positions)."""
    out = {}
    rng = np.random.default_rng(14)
    systems = {
        # cubic ABX3 3x3x3, a = 6.2, jittered: the 135-atom system of the benchmark configs
        "perov": None,
        # a triclinic cell with a short axis (images up to 2 away)
        "tric": (np.array([[7.5, 0.0, 0.0], [1.9, 8.1, 0.0], [-1.2, 2.3, 9.4]], np.float32), 60),
    }
    for tag, spec in systems.items():
        if spec is None:
            frac_cell = np.array([[0, 0, 0], [.5, .5, .5], [.5, .5, 0], [.5, 0, .5], [0, .5, .5]])
            grid = np.array([[i, j, k] for i in range(3) for j in range(3) for k in range(3)], float)
            frac = (grid[:, None, :] + frac_cell[None, :, :]).reshape(-1, 3) / 3.0
            cell = (np.eye(3) * 18.6).astype(np.float32)
            pos = frac @ cell.astype(np.float64) + rng.normal(0, 0.05, frac.shape)
        else:
            cell, n = spec
            pos = rng.uniform(0, 1, (n, 3)) @ cell.astype(np.float64) + rng.normal(0, 0.3, (n, 3))
        pos32 = pos.astype(np.float32)
        cell_t = torch.from_numpy(cell)
        inv = torch.linalg.inv(cell_t)
        p = torch.from_numpy(pos32)
        frac_un = (p.unsqueeze(-1) * inv.unsqueeze(-3)).sum(dim=-2)
        wraps = torch.floor(frac_un).to(torch.int32)
        wrapped = ((frac_un - wraps.float()).unsqueeze(-1) * cell_t.unsqueeze(-3)).sum(dim=-2)
        wrapped64 = wrapped.double().numpy()
        cell64 = cell.astype(np.float64)
        N = pos.shape[0]
        # dense candidate lists at rc + skin (6 + 2), full list, every image in reach
        rc, cand = 6.0, 8.0
        heights = abs(np.linalg.det(cell64)) / np.array(
            [np.linalg.norm(np.cross(cell64[(k + 1) % 3], cell64[(k + 2) % 3])) for k in range(3)])
        reach = [int(np.ceil(cand / h)) + 1 for h in heights]
        rows = [[] for _ in range(N)]
        for ix in range(-reach[0], reach[0] + 1):
            for iy in range(-reach[1], reach[1] + 1):
                for iz in range(-reach[2], reach[2] + 1):
                    shift = np.array([ix, iy, iz], float) @ cell64
                    d = np.linalg.norm(wrapped64[None, :, :] + shift - wrapped64[:, None, :], axis=-1)
                    for i, j in zip(*np.nonzero(d < cand)):
                        if i != j or (ix, iy, iz) != (0, 0, 0):
                            rows[i].append((j, ix, iy, iz))
        bmax = max(len(r) for r in rows)
        bmax = (bmax + 15) // 16 * 16
        nm = np.full((N, bmax), N, np.int32)
        ns = np.zeros((N, bmax, 3), np.int32)
        nn = np.zeros(N, np.int32)
        for i, r in enumerate(rows):
            rng.shuffle(r)  # candidate order must not matter
            nn[i] = len(r)
            for k, (j, ix, iy, iz) in enumerate(r):
                nm[i, k] = j
                ns[i, k] = (ix, iy, iz)
        t = dict(nm=torch.from_numpy(nm), ns=torch.from_numpy(ns), nn=torch.from_numpy(nn))
        wrap_delta = torch.zeros(N, 3, dtype=torch.int32)
        counts = torch.zeros(N, dtype=torch.int32)
        iso = torch.zeros(1, dtype=torch.int32)
        dummy_i = torch.zeros(1, dtype=torch.int32)
        dummy_b = torch.zeros(1, dtype=torch.bool)
        block = 1 << (bmax - 1).bit_length()
        fcb._count_neighbors_kernel[(N,)](
            wrapped, cell_t, t["nm"], t["ns"], t["nn"], wrap_delta, counts, counts, iso, dummy_i, N,
            dummy_b, dummy_b, dummy_i, N=N, BMAX=bmax, BLOCK=block, EDGE_CUTOFF2=rc * rc, LINE_CUTOFF2=0.0,
            HAS_SHORT=False)
        offsets = torch.zeros(N + 1, dtype=torch.int64)
        offsets[1:] = torch.cumsum(counts, 0)
        E = int(offsets[-1])
        center = torch.zeros(E, dtype=torch.int64)
        neighbor = torch.zeros(E, dtype=torch.int64)
        images = torch.zeros(E, 3, dtype=torch.int32)
        dist = torch.zeros(E, dtype=torch.float32)
        fcb._materialize_neighbors_kernel[(N,)](
            wrapped, cell_t, t["nm"], t["ns"], t["nn"], wrap_delta, offsets, center, neighbor, images, dist,
            counts, counts, N, dummy_b, dummy_b, dummy_i, N=N, BMAX=bmax, E_CAP=E, BLOCK=block,
            EDGE_CUTOFF2=rc * rc, LINE_CUTOFF2=0.0, HAS_SHORT=False)
        max_image = 12
        radix = 2 * max_image + 1
        key = ((center * N + neighbor) * radix**3 + (images[:, 0].long() + max_image) * radix * radix
               + (images[:, 1].long() + max_image) * radix + images[:, 2].long() + max_image)
        order = torch.argsort(key)
        out[f"nbr_{tag}_cell"] = cell
        out[f"nbr_{tag}_positions"] = pos32
        out[f"nbr_{tag}_wrapped"] = wrapped.numpy()
        out[f"nbr_{tag}_wraps"] = wraps.numpy()
        out[f"nbr_{tag}_cand_matrix"] = nm
        out[f"nbr_{tag}_cand_shifts"] = ns
        out[f"nbr_{tag}_cand_count"] = nn
        out[f"nbr_{tag}_counts"] = counts.numpy()
        out[f"nbr_{tag}_edges"] = np.stack([center[order].numpy(), neighbor[order].numpy()], 1)
        out[f"nbr_{tag}_images"] = images[order].numpy()
        out[f"nbr_{tag}_dist"] = dist[order].numpy()
        out[f"nbr_{tag}_cutoffs"] = np.array([rc, cand])
    return out


def bond_graph_cases(torch, fcb):
    """The reference's fixed-capacity MatRIS bond graph (a builder with a line graph): the re-filter with
    short flags (``_count_neighbors_kernel`` / ``_materialize_neighbors_kernel`` with ``LINE_CUTOFF2``,
    fixed_capacity_builder.py:98/:189), the padding rows (``_pad_edges_kernel`` :292, sink atoms;
    ``_pad_loop_pairs_kernel`` :397, far self-loops), then the builder's own ``_materialize_pairs`` (:2001),
    ``_materialize_line_graph`` (:2101, with ``_line_graph_kernel`` :681) and
    ``_substitute_overflow_topology`` (:2163) over the overflow topology of ``_allocate_overflow_topology``
    (:1474), run as unbound methods on a stand-in holding the builder's buffers. Candidates: the dense
    list within rc + 2 of the wrapped positions. Cases: both paddings with room, a triplet overflow
    (t_capacity one short) and an edge overflow (e_capacity equal to the edge count: no padding pair)."""
    from types import SimpleNamespace

    from fastmd.graph.fixed_capacity_builder import PaddingRule, self_loop_padding

    out = {}
    rng = np.random.default_rng(31)
    frac_cell = np.array([[0, 0, 0], [.5, .5, .5], [.5, .5, 0], [.5, 0, .5], [0, .5, .5]])
    grid = np.array([[i, j, k] for i in range(3) for j in range(3) for k in range(3)], float)
    perov_cell = (np.eye(3) * 18.6).astype(np.float32)
    perov = ((grid[:, None, :] + frac_cell[None, :, :]).reshape(-1, 3) / 3.0) @ perov_cell.astype(np.float64)
    perov = (perov + rng.normal(0, 0.05, perov.shape)).astype(np.float32)
    tric_cell = np.array([[7.5, 0.0, 0.0], [1.9, 8.1, 0.0], [-1.2, 2.3, 9.4]], np.float32)
    tric = (rng.uniform(0, 1, (40, 3)) @ tric_cell.astype(np.float64) + rng.normal(0, 0.3, (40, 3))).astype(np.float32)
    # (positions, cell, padding, n_dummy, extra undirected pairs, extra triplets)
    cases = {"perov_sink": (perov, perov_cell, "sink_atoms", 64, 37, 123),
             "perov_loop": (perov, perov_cell, "far_self_loops", 0, 20, 64),
             "perov_sink_tover": (perov, perov_cell, "sink_atoms", 16, 5, -1),
             "perov_loop_eover": (perov, perov_cell, "far_self_loops", 0, 0, 50),
             "tric_sink": (tric, tric_cell, "sink_atoms", 8, 11, 9)}
    rc, lrc, cand = 6.0, 4.5, 8.0
    for tag, (pos32, cell, padding, n_dummy, extra_u, extra_t) in cases.items():
        cell_t = torch.from_numpy(cell)
        inv = torch.linalg.inv(cell_t.double()).float()
        p = torch.from_numpy(pos32)
        frac_un = (p.unsqueeze(-1) * inv.unsqueeze(-3)).sum(dim=-2)
        wraps = torch.floor(frac_un).to(torch.int32)
        wrapped = ((frac_un - wraps.float()).unsqueeze(-1) * cell_t.unsqueeze(-3)).sum(dim=-2)
        wrapped64, cell64, N = wrapped.double().numpy(), cell.astype(np.float64), pos32.shape[0]
        heights = abs(np.linalg.det(cell64)) / np.array(
            [np.linalg.norm(np.cross(cell64[(k + 1) % 3], cell64[(k + 2) % 3])) for k in range(3)])
        reach = [int(np.ceil(cand / h)) + 1 for h in heights]
        rows = [[] for _ in range(N)]
        for ix in range(-reach[0], reach[0] + 1):
            for iy in range(-reach[1], reach[1] + 1):
                for iz in range(-reach[2], reach[2] + 1):
                    shift = np.array([ix, iy, iz], float) @ cell64
                    d = np.linalg.norm(wrapped64[None, :, :] + shift - wrapped64[:, None, :], axis=-1)
                    for i, j in zip(*np.nonzero(d < cand)):
                        if i != j or (ix, iy, iz) != (0, 0, 0):
                            rows[i].append((j, ix, iy, iz))
        bmax = (max(len(r) for r in rows) + 15) // 16 * 16
        nm = np.full((N, bmax), N, np.int32)
        ns = np.zeros((N, bmax, 3), np.int32)
        nn = np.zeros(N, np.int32)
        for i, r in enumerate(rows):
            rng.shuffle(r)
            nn[i] = len(r)
            for k, (j, ix, iy, iz) in enumerate(r):
                nm[i, k], ns[i, k] = j, (ix, iy, iz)
        nm_t, ns_t, nn_t = torch.from_numpy(nm), torch.from_numpy(ns), torch.from_numpy(nn)
        wrap_delta = torch.zeros(N, 3, dtype=torch.int32)
        dummy_i, dummy_b = torch.zeros(1, dtype=torch.int32), torch.zeros(1, dtype=torch.bool)
        block = 1 << (bmax - 1).bit_length()
        edge_counts = torch.zeros(N, dtype=torch.int64)
        short_counts = torch.zeros(N, dtype=torch.int64)
        iso = torch.zeros(1, dtype=torch.int32)
        fcb._count_neighbors_kernel[(N,)](
            wrapped, cell_t, nm_t, ns_t, nn_t, wrap_delta, edge_counts, short_counts, iso, dummy_i, N, dummy_b,
            dummy_b, dummy_i, N=N, BMAX=bmax, BLOCK=block, EDGE_CUTOFF2=rc * rc, LINE_CUTOFF2=lrc * lrc)
        total = int(edge_counts.sum())
        u_cap = total // 2 + extra_u
        e_cap = 2 * u_cap
        t_real = int((short_counts * (short_counts - 1)).sum())
        t_cap = t_real + extra_t
        b = SimpleNamespace(n_real=N, n_dummy=n_dummy, u_capacity=u_cap, e_capacity=e_cap, t_capacity=t_cap,
                            buffer_max=bmax, device=torch.device("cpu"), sort_key_dtype=torch.int64,
                            sort_key_max_image=10, ghosts=None, _ghost_edges=0)
        b.edge_ids = torch.arange(e_cap, dtype=torch.int64)
        b.u_ids = torch.arange(u_cap, dtype=torch.int64)
        b.triplet_ids = torch.arange(t_cap, dtype=torch.int64)
        b._pad_loop = (None if padding == "sink_atoms"
                       else self_loop_padding(PaddingRule("far_self_loops"), cell_t, rc))
        b.edge_counts, b.short_counts = edge_counts, short_counts
        b.edge_offsets = torch.zeros(N + 1, dtype=torch.int64)
        b.edge_offsets[1:] = torch.cumsum(edge_counts, 0)
        b.short_offsets = torch.zeros(N + 1, dtype=torch.int64)
        b.pair_offsets = torch.zeros(N + 1, dtype=torch.int64)
        b.short_edge_matrix = torch.zeros((N, bmax), dtype=torch.int32)
        b.center = torch.zeros(e_cap, dtype=torch.int32)
        b.neighbor = torch.zeros(e_cap, dtype=torch.int32)
        b.images = torch.zeros((e_cap, 3), dtype=torch.int32)
        b.distances = torch.zeros(e_cap, dtype=torch.float32)
        b.short_flags = torch.zeros(e_cap, dtype=torch.bool)
        b.directed2undirected = torch.zeros(e_cap, dtype=torch.int32)
        b.undirected2directed = torch.zeros(u_cap, dtype=torch.int32)
        b.line_graph = torch.zeros((t_cap, 5), dtype=torch.int32)
        b._u2d_scatter = torch.empty(u_cap + e_cap, dtype=torch.int64)
        b._short_scatter = torch.empty(N * bmax + e_cap, dtype=torch.int64)
        b._overflow = torch.zeros(1, dtype=torch.bool)
        b._invalid_pairs = torch.zeros(1, dtype=torch.bool)
        b._candidate_valid = torch.ones(1, dtype=torch.bool)
        fcb._materialize_neighbors_kernel[(N,)](
            wrapped, cell_t, nm_t, ns_t, nn_t, wrap_delta, b.edge_offsets, b.center, b.neighbor, b.images,
            b.distances, b.short_flags, b.short_edge_matrix, N, dummy_b, dummy_b, dummy_i, N=N, BMAX=bmax,
            E_CAP=e_cap, BLOCK=block, EDGE_CUTOFF2=rc * rc, LINE_CUTOFF2=lrc * lrc)
        grid = ((e_cap + 255) // 256,)
        if b._pad_loop is None:
            fcb._pad_edges_kernel[grid](b.edge_offsets[-1:], b.center, b.neighbor, b.images, b.distances,
                                        b.short_flags, N=N, N_DUMMY=n_dummy, E_CAP=e_cap, BLOCK=256)
        else:
            image, length, _ = b._pad_loop
            fcb._pad_loop_pairs_kernel[grid](b.edge_offsets[-1:], b.center, b.neighbor, b.images, b.distances,
                                             b.short_flags, *image, length, N=N, E_CAP=e_cap, BLOCK=256)
        cls = fcb.FixedCapacityGraphBuilder
        cls._allocate_overflow_topology(b)
        cls._materialize_pairs(b)
        cls._materialize_line_graph(b)
        cls._substitute_overflow_topology(b)
        out.update({f"bg_{tag}_positions": pos32, f"bg_{tag}_cell": cell,
                    f"bg_{tag}_meta": np.array([N, n_dummy, u_cap, t_cap, total, t_real,
                                                int(padding == "sink_atoms")], dtype=np.int64),
                    f"bg_{tag}_cutoffs": np.array([rc, lrc, cand]),
                    f"bg_{tag}_pad_image": np.array(b._pad_loop[0] if b._pad_loop else (0, 0, 0), np.int32),
                    f"bg_{tag}_center": b.center.numpy(), f"bg_{tag}_neighbor": b.neighbor.numpy(),
                    f"bg_{tag}_images": b.images.numpy(), f"bg_{tag}_d2u": b.directed2undirected.numpy(),
                    f"bg_{tag}_u2d": b.undirected2directed.numpy(), f"bg_{tag}_line_graph": b.line_graph.numpy(),
                    f"bg_{tag}_short_flags": b.short_flags.numpy(),
                    f"bg_{tag}_flags": np.array([bool(b._overflow), bool(b._invalid_pairs)], dtype=np.int64)})
    return out


def float64_cases(torch, fcb):
    """The float64 edges-only build's prologue, ``_float64_prologue_kernel`` (fixed_capacity_builder.py:464):
    float32 wrap of the rounded coordinates, the float64 model positions (coordinates minus the same whole
    lattice vectors of the float64 cell), the wrap delta and the skin test against a refresh snapshot, on
    a triclinic cell and the perovskite's cubic one, coordinates spread over several lattice images."""
    out = {}
    rng = np.random.default_rng(41)
    cells = {"tric": np.array([[7.5, 0.0, 0.0], [1.9, 8.1, 0.0], [-1.2, 2.3, 9.4]]),
             "cubic": np.eye(3) * 18.6}
    for tag, cell64 in cells.items():
        n = 97
        frac = rng.uniform(-1.5, 2.5, (n, 3))
        ref64 = frac @ cell64
        pos64 = ref64 + rng.normal(0.0, 0.15, (n, 3))  # some atoms cross a cell face since the refresh
        if tag == "cubic":
            pos64[5] += 0.9 * cell64[0]  # and one moves far beyond half the skin
        cell32 = torch.from_numpy(cell64.astype(np.float32))
        inv32 = torch.linalg.inv(cell32.double()).float()
        q_ref = torch.from_numpy(ref64.astype(np.float32))
        ref_wraps = torch.floor((q_ref.unsqueeze(-1) * inv32.unsqueeze(-3)).sum(dim=-2)).to(torch.int32)
        frac_out = torch.zeros(n, 3)
        wrapped = torch.zeros(n, 3)
        wrap_delta = torch.zeros(n, 3, dtype=torch.int32)
        model = torch.zeros(n, 3, dtype=torch.float64)
        max_disp = torch.zeros(1)
        valid = torch.zeros(1, dtype=torch.bool)
        iso = torch.zeros(1, dtype=torch.int32)
        skin = 2.0
        fcb._float64_prologue_kernel[(1,)](
            torch.from_numpy(pos64), inv32.contiguous(), cell32.contiguous(), torch.from_numpy(cell64).contiguous(),
            q_ref, ref_wraps, torch.ones(1, dtype=torch.bool), frac_out, wrapped, wrap_delta, model, max_disp, valid,
            iso, skin + 1.0e-6, N=n, BLOCK=128)
        out.update({f"f64_{tag}_cell": cell64, f"f64_{tag}_positions": pos64, f"f64_{tag}_reference": ref64,
                    f"f64_{tag}_inv32": inv32.numpy(), f"f64_{tag}_ref_wraps": ref_wraps.numpy(),
                    f"f64_{tag}_frac": frac_out.numpy(), f"f64_{tag}_wrapped": wrapped.numpy(),
                    f"f64_{tag}_wrap_delta": wrap_delta.numpy(), f"f64_{tag}_model_positions": model.numpy(),
                    f"f64_{tag}_max_displacement": max_disp.numpy(), f"f64_{tag}_candidate_valid": valid.numpy(),
                    f"f64_{tag}_skin": np.array([skin])})
    return out


def padding_cases(torch, fcb):
    """The edges-only padding rows: ``_pad_self_loops_kernel`` (fixed_capacity_builder.py:324) with the far
    self-loop image of a cubic 18.6 A cell (no override) and with image 0 and the exact-rc override vector
    (6, 0, 0) at a 6 A cutoff (HAS_OVERRIDE), for 2,054 real edges of 2,200 rows over 135 atoms (the config-1
    count)."""
    out = {}
    total, e_cap, n = 2054, 2200, 135
    for tag, image, vector, override in (("far", (1, 0, 0), (0.0, 0.0, 0.0), False),
                                         ("exact_rc", (0, 0, 0), (6.0, 0.0, 0.0), True)):
        center = torch.full((e_cap,), -7, dtype=torch.int32)
        neighbor = torch.full((e_cap,), -7, dtype=torch.int32)
        images = torch.full((e_cap, 3), -7, dtype=torch.int32)
        vec = torch.full((e_cap, 3), -7.0)
        fcb._pad_self_loops_kernel[((e_cap + 255) // 256,)](
            torch.tensor([total], dtype=torch.int64), center, neighbor, images, vec if override else images,
            *image, *vector, torch.zeros(1, dtype=torch.int32), N=n, E_CAP=e_cap, BLOCK=256, HAS_OVERRIDE=override)
        out.update({f"pad_{tag}_meta": np.array([total, e_cap, n], dtype=np.int64),
                    f"pad_{tag}_center": center.numpy(), f"pad_{tag}_neighbor": neighbor.numpy(),
                    f"pad_{tag}_images": images.numpy(), f"pad_{tag}_override": vec.numpy(),
                    f"pad_{tag}_image": np.array(image, np.int32), f"pad_{tag}_vector": np.array(vector, np.float32)})
    return out


def radial_cases(torch):
    """The reference's radial basis (fastmd/models/matris/basis_function.py:139 BesselExpansion with the
    PolynomialEnvelope of :31) at the MACE setting (8 functions, rc 6, p 5) and MatRIS's (7, 6, 8)."""
    from fastmd.models.matris.basis_function import BesselExpansion

    d = torch.linspace(0.35, 6.4, 977, dtype=torch.float32)
    out = {"radial_d": d.numpy()}
    for tag, (n, rc, p) in {"mace": (8, 6.0, 5), "matris": (7, 6.0, 8)}.items():
        module = BesselExpansion(num_radial=n, cutoff=rc, envelope_exponent=p)
        out[f"radial_{tag}"] = module(d).detach().numpy()
        out[f"radial_{tag}_params"] = np.array([n, rc, p], dtype=np.float64)
    return out


def main(reference: str, only: list[str]) -> None:
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, str(HERE))
    _install_stubs()
    sys.path.insert(0, reference)
    import torch

    import fastmd.execution.gpu_nhc as gpu_nhc
    import fastmd.graph.neighbor_list_backend as backend

    # The re-filter kernels are defined only when the candidate backend (nvalchemiops, absent here)
    # imports; they do not call it, so its import check is bypassed for this script.
    backend.require = lambda: None
    import fastmd.graph.fixed_capacity_builder as fcb
    import fastmd.models.matris.op.triton_csr_segment_sum as cs
    import fastmd.models.matris.op.triton_gather_cat as gc
    import fastmd.models.matris.op.triton_segment_attention as sa
    import fastmd.engine.kernels.decomposed_indexed_cat_silu_linear as di
    import fastmd.graph.gpu_graph_builder as ggb
    import fastmd.models.matris.op.triton_gated_ln as gl
    import fastmd.models.matris.op.triton_directed_pair_aggregate as pa
    import fastmd.models.matris.op.triton_residual_add as ra
    import fastmd.models.matris.op.triton_line_envelope as le
    import fastmd.engine.kernels.triton_wide_gemm as wg

    fixtures = {
        "gather_cat": lambda: gather_cat_cases(torch, gc),
        "segment_sum": lambda: segment_sum_cases(torch, cs),
        "nhc": lambda: nhc_cases(torch, gpu_nhc),
        "neighbors": lambda: neighbor_cases(torch, fcb),
        "radial": lambda: radial_cases(torch),
        "segment_attention": lambda: segment_attention_cases(torch, sa),
        "gather_add_silu": lambda: gather_add_silu_cases(torch, di),
        "line_graph": lambda: pairs_line_graph_cases(torch, ggb),
        "gated_ln": lambda: gated_ln_cases(torch, gl),
        "pair_aggregate": lambda: pair_aggregate_cases(torch, pa),
        "residual_add": lambda: residual_add_cases(torch, ra),
        "bond_graph": lambda: bond_graph_cases(torch, fcb),
        "float64": lambda: float64_cases(torch, fcb),
        "padding": lambda: padding_cases(torch, fcb),
        "matris": lambda: matris_cases(torch),
        "line_envelope": lambda: line_envelope_cases(torch, le),
        "wide_gemm": lambda: wide_gemm_cases(torch, wg),
    }
    for name, make in fixtures.items():
        if not only or name in only:
            np.savez_compressed(HERE / f"{name}.npz", **make())
    for path in sorted(HERE.glob("*.npz")):
        print(path.name, path.stat().st_size)


if __name__ == "__main__":
    # make_golden.py <reference-root> [fixture ...]: every fixture unless some are named
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden.py <reference-root> [fixture ...]")
    main(sys.argv[1], sys.argv[2:])
