"""The operator surface the MatRIS model sites call, routed to this build's kernels.

Mirrors ``OpDispatcher`` of fastmd/engine/dispatch.py:142 (the P=1 operator selection, attached to a
processed batch as ``graph["_ops"]`` by ``attach_dispatcher`` :115): the same method names, argument
meanings and graph-dict cache keys, so a model site written against the reference's dispatcher runs
unchanged. Where the reference chooses between a fused Triton kernel and a PyTorch fallback by policy
switches and row thresholds, every method here runs the CUDA kernel of libfastmd_b200.so; the eligibility
predicates (``use_*``) answer whether the tensors meet the kernel's shape rules, and inputs that do not
raise instead of falling back (there is no CPU path). The weighted segment sum is the deterministic CSR
sum (the reference's fallback is an atomic scatter; the sums agree to FP32 rounding).

* ``pair_expand`` / ``pair_average`` (:210, :235) -> ``pair_aggregate`` over the cached ``[U, 2]`` pair
  index ``graph["_directed2undirected_pair_index"]`` (:633);
* ``residual`` (:265) -> ``residual_add`` (frozen weight only);
* ``segment_sum_graph`` / ``segment_sum`` (:349, :371) -> ``ops.csr_segment_sum`` / ``ops.aggregate`` over the
  side CSRs ``graph[f"_{side}_segment_sum_csr"]`` that ``prepare_segment_csr`` (:311) stores;
* ``segment_attention`` (:421) -> ``segment_attention`` / ``paired_segment_attention`` over the CSRs cached as
  ``graph[f"_{side}_segment_attention_perm"/"_offsets"]`` (:603);
* ``gather`` / ``gather_cat`` (:515, :547) -> the gather-cat kernel.
"""
from __future__ import annotations

import torch
from torch import Tensor

from . import ops
from .pair_aggregate import directed_pair_average, undirected_pair_expand
from .residual_add import residual_add
from .segment_attention import paired_segment_attention, segment_attention


def _directed_pair_index(graph: dict, directed2undirected: Tensor) -> Tensor:
    """``[U, 2]`` directed rows of every pair (argsort of the pair id of each directed row), cached in
    ``graph`` under the reference's key (dispatch.py:633)."""
    key = "_directed2undirected_pair_index"
    pair_index = graph.get(key)
    if pair_index is None:
        pair_index = torch.argsort(directed2undirected, stable=True).reshape(graph["num_undirected"], 2).contiguous()
        graph[key] = pair_index
    return pair_index


def _attention_csr(graph: dict, side: str, segment: Tensor, num_segment: int, identity: bool):
    """(perm, offsets, identity) of one attention side, cached under the reference's keys (dispatch.py:603):
    an identity CSR (rows sorted by segment) from the cached offsets or counts, else perm/offsets of
    ``segment``."""
    perm_key, off_key = f"_{side}_segment_attention_perm", f"_{side}_segment_attention_offsets"
    if identity:
        off = graph.get(off_key)
        if off is None:
            counts = graph[f"_{side}_segment_attention_counts"]
            off = torch.cat((counts.new_zeros(1), counts.cumsum(0))).to(torch.int64)
            graph[off_key] = off
        return None, off, True
    perm, off = graph.get(perm_key), graph.get(off_key)
    if perm is None or off is None:
        perm, off = ops.segment_csr(segment, num_segment)
        graph[perm_key], graph[off_key] = perm, off
    return perm, off, False


class OpDispatcher:
    """The P=1 operator surface of fastmd/engine/dispatch.py:142 on this build's kernels.

    ``paired_attention``: both attention sides of one graph sharing their value rows (tensor identity) run
    as one paired attention (the reference's ``MATRIS_FUSED_PAIRED_SEGMENT_ATTENTION``).
    ``identity_target_csr``: the target side's rows are certified sorted by segment per graph kind
    (``{"atom", "line"}``), so its CSR is the identity with offsets from the cached counts (the
    reference's ``..._SORTED_TARGET_CSR`` with a layout that certifies it).
    """

    def __init__(self, *, paired_attention: bool = True, identity_target_csr=()):
        self.paired_attention = bool(paired_attention)
        self.identity_csr = {kind: kind in set(identity_target_csr) for kind in ("atom", "line")}
        unknown = set(identity_target_csr) - {"atom", "line"}
        if unknown:
            raise ValueError(f"identity_target_csr: graph kinds are 'atom' and 'line', got {sorted(unknown)}")
        self.segment_sum_csr_enabled = True

    def __repr__(self) -> str:
        kinds = [k for k, v in self.identity_csr.items() if v]
        return f"OpDispatcher(paired_attention={self.paired_attention}, identity_target_csr={kinds})"

    # ------------------------------------------------------------ pair maps

    def pair_expand(self, data: Tensor, directed2undirected: Tensor, graph: dict) -> Tensor:
        """``data[d2u]``: undirected rows ``[U, D]`` -> directed rows ``[2U, D]``."""
        return undirected_pair_expand(data, _directed_pair_index(graph, directed2undirected),
                                      directed2undirected.numel())

    def pair_average(self, data: Tensor, directed2undirected: Tensor, graph: dict) -> Tensor:
        """Mean of the two directed rows of every pair: ``[2U, D]`` -> ``[U, D]``."""
        if directed2undirected.numel() != 2 * graph["num_undirected"]:
            raise ValueError(f"directed2undirected holds {directed2undirected.numel()} rows for "
                             f"{graph['num_undirected']} undirected pairs")
        return directed_pair_average(data, _directed_pair_index(graph, directed2undirected))

    # ------------------------------------------------------------ residuals

    def residual(self, delta: Tensor, residual: Tensor, weight: Tensor) -> Tensor:
        """``delta + weight * residual`` with a frozen ``weight`` (no weight gradient is formed)."""
        if weight.requires_grad:
            raise ValueError("residual: this build's residual add takes a frozen weight (requires_grad=False)")
        return residual_add(delta, residual, weight)

    def gated_ln_residual(self) -> tuple[bool, int]:
        """(enabled, min_rows) of the fused gated-LN residual epilogue (``gated_ln.fused_gated_ln_residual``)."""
        return True, 0

    # ------------------------------------------------------------ segment sums

    def use_csr_segment_sum(self, value: Tensor, segment: Tensor, weight: Tensor | None) -> bool:
        """Whether the tensors meet the CSR segment sum's rules (dispatch.py:335)."""
        if not (value.is_cuda and segment.is_cuda and value.dim() == 2):
            return False
        if weight is not None and not (weight.is_cuda and weight.shape == value.shape and weight.dtype == value.dtype):
            return False
        return segment.dim() == 1 and segment.numel() == value.shape[0]

    def prepare_segment_csr(self, graph: dict, num_segment: int) -> None:
        """Store ``graph[f"_{side}_segment_sum_csr"] = (perm, offsets, identity, -1)`` for both sides,
        sharing the attention CSR cache (the identity CSR for a certified sorted target side)."""
        kind = "atom" if graph.get("_topology_graph_kind") == "atom" else "line"
        for side in ("source", "target"):
            identity = (side == "target" and self.identity_csr[kind]
                        and (f"_{side}_segment_attention_counts" in graph
                             or f"_{side}_segment_attention_offsets" in graph))
            perm, off, identity = _attention_csr(graph, side, graph[f"{side}_index"], num_segment, identity)
            graph[f"_{side}_segment_sum_csr"] = (perm, off, identity, -1)

    def segment_csr(self, graph: dict, side: str, segment: Tensor, num_segment: int):
        """(perm, int64 offsets, identity, skip_segment) of ``side`` of ``graph``."""
        csr = graph.get(f"_{side}_segment_sum_csr")
        if csr is None:
            self.prepare_segment_csr(graph, num_segment)
            csr = graph[f"_{side}_segment_sum_csr"]
        return csr

    def segment_sum_graph(self, value: Tensor, segment: Tensor, num_segment: int, graph: dict, side: str, *,
                          weight: Tensor | None = None, bin_count: Tensor | None = None) -> Tensor:
        """``segment_sum`` over ``side`` (``"source"`` / ``"target"``) of ``graph`` on the side's CSR."""
        if self.use_csr_segment_sum(value, segment, weight):
            perm, off, identity, skip_segment = self.segment_csr(graph, side, segment, num_segment)
            return ops.csr_segment_sum(value, segment, num_segment, perm, off, identity, weight=weight,
                                       skip_segment=skip_segment)
        return self.segment_sum(value, segment, num_segment, weight=weight, bin_count=bin_count)

    def segment_sum(self, value: Tensor, segment: Tensor, num_segment: int, *, weight: Tensor | None = None,
                    bin_count: Tensor | None = None) -> Tensor:
        """``sum_{i in segment s} [weight_i *] value_i`` for ``num_segment`` segments (deterministic)."""
        if weight is None:
            return ops.aggregate(value, segment, bin_count, average=False, num_segment=num_segment)
        return ops.csr_segment_sum(value, segment, num_segment, weight=weight)

    # ------------------------------------------------------------ attention

    def use_segment_attention(self, logits: Tensor, value: Tensor) -> bool:
        """Whether the tensors meet the fused attention's rules (dispatch.py:410)."""
        return logits.is_cuda and value.is_cuda and logits.shape == value.shape and logits.dim() == 2

    def segment_attention(self, source_alpha_0: Tensor, source_rows: Tensor, source_node_index: Tensor,
                          target_alpha_0: Tensor, target_rows: Tensor, target_node_index: Tensor, num_segment: int,
                          graph: dict) -> tuple[Tensor, Tensor]:
        """Channel-wise segment softmax attention of both sides of one graph: paired when both sides share
        their value rows (tensor identity), else one attention per side."""
        kind = "atom" if graph.get("_topology_graph_kind") == "atom" else "line"
        s_perm, s_off, s_id = _attention_csr(graph, "source", source_node_index, num_segment, False)
        t_perm, t_off, t_id = _attention_csr(graph, "target", target_node_index, num_segment, self.identity_csr[kind])
        if self.paired_attention and source_rows is target_rows:
            return paired_segment_attention(source_alpha_0, target_alpha_0, source_rows, source_node_index,
                                            target_node_index, num_segment, s_perm, s_off, t_perm, t_off, s_id, t_id)
        return (segment_attention(source_alpha_0, source_rows, source_node_index, num_segment, s_perm, s_off, s_id),
                segment_attention(target_alpha_0, target_rows, target_node_index, num_segment, t_perm, t_off, t_id))

    # ------------------------------------------------------------ gathers

    def gather(self, value: Tensor, indices: Tensor) -> Tensor:
        """``value[indices]`` (rows), deterministic gradient."""
        return ops.gather_cat([(value, indices)])

    def use_gather_cat(self, aligned: Tensor, gathered: Tensor) -> bool:
        """Whether the 3-part aligned gather-cat applies (equal widths, 2-D CUDA tensors)."""
        return (aligned.is_cuda and gathered.is_cuda and aligned.dim() == 2 and gathered.dim() == 2
                and aligned.shape[1] == gathered.shape[1])

    def use_gather_cat4(self, aligned: Tensor, gathered_a: Tensor, gathered_b: Tensor) -> bool:
        """Whether the 4-part gather-cat applies (mixed widths run too: ``ops.gather_cat`` takes any)."""
        return all(t.is_cuda and t.dim() == 2 for t in (aligned, gathered_a, gathered_b))

    def gather_cat(self, aligned: Tensor, gathered, indices) -> Tensor:
        """Fused ``cat([aligned, gathered_k[indices_k]...], 1)`` (3 or 4 parts)."""
        if len(gathered) == 1:
            return ops.aligned_gather_cat3(aligned, gathered[0], indices[0], indices[1])
        if self.use_gather_cat(aligned, gathered[0]) and aligned.shape[1] == gathered[1].shape[1]:
            return ops.aligned_gather_cat4(aligned, gathered[0], indices[0], gathered[1], indices[1], indices[2])
        return ops.gather_cat([(aligned, None), (gathered[0], indices[0]), (gathered[1], indices[1]),
                               (gathered[1], indices[2])])


def attach_dispatcher(batch_graph: dict, dispatcher: OpDispatcher | None = None) -> OpDispatcher:
    """Attach ``dispatcher`` (a default one when None) to a processed batch as the reference does
    (dispatch.py:115): ``batch_graph["_ops"]`` and the ``_ops`` of its atom and line graph dicts, and the
    side CSRs of both graphs prepared before any layer runs."""
    dispatcher = OpDispatcher() if dispatcher is None else dispatcher
    batch_graph["_ops"] = dispatcher
    atom_graph, line_graph = batch_graph["atom_graph_dict"], batch_graph["line_graph_dict"]
    atom_graph["_ops"] = dispatcher
    line_graph["_ops"] = dispatcher
    dispatcher.prepare_segment_csr(atom_graph, atom_graph["num_segment"])
    if "target_index" in line_graph:
        dispatcher.prepare_segment_csr(line_graph, atom_graph["num_undirected"])
    return dispatcher


__all__ = ["OpDispatcher", "attach_dispatcher"]
