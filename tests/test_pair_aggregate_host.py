"""Host-side logic of the pair-aggregation surface: the admission check and the shape errors of
fastmd/models/matris/op/triton_directed_pair_aggregate.py (:261, :292), no kernel call."""
import pytest
import torch

from fastmd_b200.pair_aggregate import directed_pair_average, pair_index_bijection_reason, undirected_pair_expand


def test_bijection_reasons():
    assert pair_index_bijection_reason([[0, 1]], 2) == "not_tensor"
    assert pair_index_bijection_reason(torch.zeros(3, dtype=torch.int64), 6).startswith("pair_index_shape")
    assert pair_index_bijection_reason(torch.zeros(2, 2), 4).startswith("index_dtype")
    assert pair_index_bijection_reason(torch.tensor([[0, 1]]), 5).startswith("num_directed")
    assert pair_index_bijection_reason(torch.empty(0, 2, dtype=torch.int64), 0) is None
    assert pair_index_bijection_reason(torch.tensor([[0, 1], [2, 4]]), 4).startswith("index_out_of_range")
    assert pair_index_bijection_reason(torch.tensor([[0, 1], [1, 2]]), 4) == "duplicate_directed_row"
    assert pair_index_bijection_reason(torch.tensor([[3, 0], [2, 1]], dtype=torch.int32), 4) is None


def test_shape_errors_before_any_kernel():
    pair = torch.tensor([[0, 1], [2, 3]])
    with pytest.raises(ValueError, match="expected 2 data row"):
        directed_pair_average(torch.zeros(5, 3), pair)
    with pytest.raises(ValueError, match=r"expected data \[rows, D\]"):
        directed_pair_average(torch.zeros(4), pair)
    with pytest.raises(ValueError, match="num_directed must be 2U"):
        undirected_pair_expand(torch.zeros(2, 3), pair, 5)
    with pytest.raises(ValueError, match="expected 1 data row"):
        undirected_pair_expand(torch.zeros(3, 3), pair, 4)


def test_cpu_tensors_raise():
    from fastmd_b200._lib import FastMDLibraryError

    with pytest.raises(FastMDLibraryError):
        directed_pair_average(torch.zeros(4, 3), torch.tensor([[0, 1], [2, 3]]))
