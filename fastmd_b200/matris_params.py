"""MatRIS hyperparameters and the parameter layout of a MatRIS checkpoint (host side, NumPy only).

``MatRISConfig`` holds the hyperparameters of the bundled MatRIS potential
(fastmd/models/matris/model.py:107-135). ``MATRIS_10M`` is the library's 10M
architecture ``OAM_10M`` (fastmd/engine/memory_admission.py:228: 10 layers,
node/edge/three-body width 128, widest MLP hidden 256, 7 radial and 7 angular
functions, cutoffs 6.0 / 4.5 A, layer norm, Fourier three-body basis, gated
MLPs) with an energy head of hidden widths (256, 256).

``parameter_shapes`` lists every tensor of a MatRIS ``state_dict`` under the
reference's own key names (the checkpoint format ``MatRIS.from_dict`` loads,
model.py:577), so a checkpoint written by the reference loads here unchanged.
``seeded_parameters`` fills that layout with seeded random values: the
benchmark configurations use random-init weights (no checkpoint download), and
the parity fixtures load the same values into the reference model.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class MatRISConfig:
    num_layers: int = 10
    node_dim: int = 128
    edge_dim: int = 128
    three_body_dim: int = 128
    energy_hidden: tuple = (256, 256)
    num_radial: int = 7
    num_angular: int = 7
    envelope_exponent: int = 8
    pairwise_cutoff: float = 6.0
    three_body_cutoff: float = 4.5
    max_elements: int = 94

    def __post_init__(self):
        if self.num_angular % 2 != 1:
            raise ValueError("num_angular must be odd (a constant plus sine and cosine pairs)")
        if not (self.node_dim == self.edge_dim == self.three_body_dim):
            raise ValueError("this build implements equal node, edge and three-body widths")
        if self.node_dim % 4:
            raise ValueError("feature widths must be multiples of 4 (16-byte rows)")

    @classmethod
    def from_reference(cls, config: dict) -> "MatRISConfig":
        """The architecture of a reference checkpoint's ``config`` dict (the constructor's keyword
        arguments, model.py:107, saved by ``MatRIS.config``); raises for the variants this build does not
        implement (norms other than LayerNorm, the SH three-body basis, plain MLP blocks, biases in the
        interaction FFNs, the smoothed edge update)."""
        kinds = {"norm_type": "layer", "three_body_expansion": "fourier", "graph_conv_mlp": "gatemlp"}
        for key, want in kinds.items():
            if str(config.get(key, want)).lower() != want:
                raise NotImplementedError(f"MatRIS {key}={config.get(key)!r}: this build implements {want!r}")
        if config.get("use_bias", False) or config.get("use_smoothed_for_delta_edge", False):
            raise NotImplementedError("MatRIS use_bias / use_smoothed_for_delta_edge are not implemented here")
        hidden = config.get("mlp_hidden_dims", (128, 128))
        hidden = (int(hidden),) if isinstance(hidden, int) else tuple(int(h) for h in hidden)
        return cls(num_layers=int(config.get("num_layers", 6)), node_dim=int(config.get("node_feat_dim", 128)),
                   edge_dim=int(config.get("edge_feat_dim", 128)),
                   three_body_dim=int(config.get("three_body_feat_dim", 128)), energy_hidden=hidden,
                   num_radial=int(config.get("num_radial", 7)), num_angular=int(config.get("num_angular", 7)),
                   envelope_exponent=int(config.get("envelope_exponent", 8)),
                   pairwise_cutoff=float(config.get("pairwise_cutoff", 6.0)),
                   three_body_cutoff=float(config.get("three_body_cutoff", 4.0)))

    @property
    def max_frequency(self) -> int:
        return (self.num_angular - 1) // 2

    def reference_kwargs(self) -> dict:
        """The reference constructor's keyword arguments for this architecture (model.py:107)."""
        return dict(num_layers=self.num_layers, node_feat_dim=self.node_dim, edge_feat_dim=self.edge_dim,
                    three_body_feat_dim=self.three_body_dim, mlp_hidden_dims=tuple(self.energy_hidden),
                    num_radial=self.num_radial, num_angular=self.num_angular, envelope_exponent=self.envelope_exponent,
                    pairwise_cutoff=self.pairwise_cutoff, three_body_cutoff=self.three_body_cutoff,
                    norm_type="layer", three_body_expansion="fourier", graph_conv_mlp="GateMLP", use_bias=False,
                    learnable_basis=True, is_intensive=True)


MATRIS_10M = MatRISConfig()


def _gated_mlp(prefix: str, fan_in: int, hidden: int, out: int) -> list:
    """A GatedMLP (functions.py:395): two MLPs ``Linear(fan_in, hidden) -> SiLU -> Linear(hidden, out)``
    with biases (core, gate) and a LayerNorm on each output."""
    rows = []
    for norm in ("gate_norm", "core_norm"):
        rows += [(f"{prefix}.{norm}.weight", (out,), "ln_w"), (f"{prefix}.{norm}.bias", (out,), "ln_b")]
    for mlp in ("mlp_core", "mlp_gate"):
        rows += [(f"{prefix}.{mlp}.layers.0.weight", (hidden, fan_in), "w"),
                 (f"{prefix}.{mlp}.layers.0.bias", (hidden,), f"b{fan_in}"),
                 (f"{prefix}.{mlp}.layers.3.weight", (out, hidden), "w"),
                 (f"{prefix}.{mlp}.layers.3.bias", (out,), f"b{hidden}")]
    return rows


def parameter_shapes(config: MatRISConfig = MATRIS_10M) -> list[tuple[str, tuple, str]]:
    """``(key, shape, kind)`` of every MatRIS checkpoint tensor (the reference's ``state_dict`` keys);
    ``kind`` selects the random initialisation."""
    C, R, A = config.node_dim, config.num_radial, config.num_angular
    rows = [("atom_embedding.embedding.weight", (config.max_elements, C), "embed"),
            ("atom_embedding.atom_swish_layer.linear.weight", (C, C), "w"),
            ("edge_embedding.pairwise_rbf_expansion.frequencies", (R,), "bessel"),
            ("edge_embedding.threebody_rbf_expansion.frequencies", (R,), "bessel"),
            ("edge_embedding.edge_linear1.weight", (C, R), "w"),
            ("edge_embedding.edge_linear2.weight", (C, C), "w"),
            ("edge_embedding.swish_layer.linear.weight", (C, C), "w"),
            ("edge_embedding.edge_init_norm.weight", (C,), "ln_w"),
            ("edge_embedding.edge_init_norm.bias", (C,), "ln_b"),
            ("three_body_embedding.expansion.frequencies", (config.max_frequency,), "fourier"),
            ("three_body_embedding.angle_embedding.weight", (C, A), "w"),
            ("three_body_embedding.swish_layer.linear.weight", (C, C), "w")]
    for b in range(config.num_layers):
        for graph in ("atom", "line"):
            p = f"interaction_block.{b}.attn_block_{graph}_graph"
            rows += [(f"{p}.node_res_weight", (1, C), "res"), (f"{p}.edge_res_weight", (1, C), "res"),
                     (f"{p}.source_weight_linear.weight", (C, C), "w"),
                     (f"{p}.target_weight_linear.weight", (C, C), "w")]
            rows += _gated_mlp(f"{p}.node_nonlinear_update", 3 * C, C, C)
            rows += _gated_mlp(f"{p}.edge_nonlinear_update", 3 * C, C, C)
        for graph in ("atom", "line"):
            p = f"interaction_block.{b}.refine_block_{graph}_graph"
            rows += [(f"{p}.node_res_weight", (1, C), "res"), (f"{p}.edge_res_weight", (1, C), "res")]
            rows += _gated_mlp(f"{p}.edge_nonlinear_update", (3 if graph == "atom" else 4) * C, C, C)
            rows += [(f"{p}.node_FFN.layers.0.weight", (C, C), "w"), (f"{p}.node_FFN.layers.3.weight", (C, C), "w"),
                     (f"{p}.edge_FFN.layers.0.weight", (C, C), "w"), (f"{p}.edge_FFN.layers.3.weight", (C, C), "w"),
                     (f"{p}.learnable_envelope.weight", (C, R if graph == "atom" else A), "w")]
    rows += [("readout_norm.weight", (C,), "ln_w"), ("readout_norm.bias", (C,), "ln_b")]
    widths = [C, *config.energy_hidden, 1]
    for i in range(len(widths) - 1):
        rows += [(f"energy_head.energy_head.layers.{3 * i}.weight", (widths[i + 1], widths[i]), "w"),
                 (f"energy_head.energy_head.layers.{3 * i}.bias", (widths[i + 1],), f"b{widths[i]}")]
    rows += [("magmom_head.magmom_head.layers.0.weight", (2 * C, C), "w"),
             ("magmom_head.magmom_head.layers.0.bias", (2 * C,), f"b{C}"),
             ("magmom_head.magmom_head.layers.3.weight", (1, 2 * C), "w"),
             ("magmom_head.magmom_head.layers.3.bias", (1,), f"b{2 * C}")]
    return rows


def seeded_parameters(config: MatRISConfig = MATRIS_10M, seed: int = 0) -> dict[str, np.ndarray]:
    """Random float32 values for every checkpoint tensor, drawn in ``parameter_shapes`` order from
    ``np.random.default_rng(seed)``: linear weights and biases uniform in +-1/sqrt(fan_in) (the
    scale of a fresh ``nn.Linear``), LayerNorm scales 1 + 0.1 N(0, 1) and shifts 0.1 N(0, 1),
    residual weights 1 + 0.1 N(0, 1), element embeddings N(0, 1), and the learnable basis
    frequencies at their initial values (n pi for the Bessel functions, n for the Fourier terms)
    times 1 + 0.02 N(0, 1)."""
    rng = np.random.default_rng(seed)
    out = {}
    for key, shape, kind in parameter_shapes(config):
        if kind == "w":
            bound = 1.0 / np.sqrt(shape[1])
            value = rng.uniform(-bound, bound, shape)
        elif kind[0] == "b" and kind[1:].isdigit():
            bound = 1.0 / np.sqrt(int(kind[1:]))
            value = rng.uniform(-bound, bound, shape)
        elif kind in ("ln_w", "res"):
            value = 1.0 + 0.1 * rng.standard_normal(shape)
        elif kind == "ln_b":
            value = 0.1 * rng.standard_normal(shape)
        elif kind == "embed":
            value = rng.standard_normal(shape)
        elif kind == "bessel":
            value = np.pi * np.arange(1, shape[0] + 1) * (1.0 + 0.02 * rng.standard_normal(shape))
        elif kind == "fourier":
            value = np.arange(1, shape[0] + 1) * (1.0 + 0.02 * rng.standard_normal(shape))
        else:  # pragma: no cover - the table above names every kind
            raise AssertionError(kind)
        out[key] = np.asarray(value, dtype=np.float32)
    return out
