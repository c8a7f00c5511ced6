"""Host logic of the OpDispatcher mirror and the residual-add wrapper (no kernel launches)."""
import pytest
import torch

from fastmd_b200 import dispatch
from fastmd_b200._lib import FastMDLibraryError
from fastmd_b200.residual_add import residual_add


def test_pair_index_is_cached_under_the_reference_key():
    d2u = torch.tensor([2, 0, 1, 0, 2, 1])
    graph = {"num_undirected": 3}
    pair = dispatch._directed_pair_index(graph, d2u)
    assert pair.tolist() == [[1, 3], [2, 5], [0, 4]]
    assert graph["_directed2undirected_pair_index"] is pair
    assert dispatch._directed_pair_index(graph, d2u) is pair


def test_identity_csr_from_cached_counts():
    graph = {"_target_segment_attention_counts": torch.tensor([2, 0, 3])}
    perm, off, identity = dispatch._attention_csr(graph, "target", torch.zeros(5, dtype=torch.int64), 3, True)
    assert perm is None and identity and off.tolist() == [0, 2, 2, 5] and off.dtype == torch.int64
    assert graph["_target_segment_attention_offsets"] is off


def test_dispatcher_options_and_errors():
    d = dispatch.OpDispatcher(identity_target_csr={"atom"})
    assert d.identity_csr == {"atom": True, "line": False}
    assert d.gated_ln_residual() == (True, 0)
    with pytest.raises(ValueError):
        dispatch.OpDispatcher(identity_target_csr={"bond"})
    x = torch.zeros(4, 8)
    with pytest.raises(ValueError, match="frozen"):
        d.residual(x, x, torch.zeros(8, requires_grad=True))
    with pytest.raises(ValueError):
        d.pair_average(x, torch.zeros(6, dtype=torch.int64), {"num_undirected": 2})
    assert not d.use_csr_segment_sum(x, torch.zeros(4, dtype=torch.int64), None)  # CPU tensors
    assert not d.use_segment_attention(x, x)


def test_residual_add_argument_errors():
    x = torch.zeros(4, 8)
    with pytest.raises(ValueError):
        residual_add(x, torch.zeros(4, 7), torch.zeros(8))
    with pytest.raises(ValueError):
        residual_add(x, x, torch.zeros(7))
    with pytest.raises(TypeError):
        residual_add(x.double(), x.double(), torch.zeros(8, dtype=torch.float64))
    with pytest.raises(FastMDLibraryError):  # no CPU path
        residual_add(x, x, torch.zeros(8))


def test_attach_dispatcher_sets_every_graph_dict(monkeypatch):
    seen = []
    monkeypatch.setattr(dispatch.OpDispatcher, "prepare_segment_csr", lambda self, g, n: seen.append((id(g), n)))
    atom, line = {"num_segment": 5, "num_undirected": 7}, {"target_index": None}
    batch = {"atom_graph_dict": atom, "line_graph_dict": line}
    d = dispatch.attach_dispatcher(batch)
    assert batch["_ops"] is d and atom["_ops"] is d and line["_ops"] is d
    assert seen == [(id(atom), 5), (id(line), 7)]
