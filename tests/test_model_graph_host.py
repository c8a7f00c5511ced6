"""Host logic of the model_graph runner: the capacity tiers of fastmd/engine/capacity_policy.py:19 and the
bucket selection of fastmd/execution/cuda_graph.py:435/:677 (no device work)."""
import pytest

from fastmd_b200.model_graph import BucketedGraphRunner, smallest_fitting_key, tier


def test_tier_is_the_next_step_with_minimum_slack():
    assert tier(0, 512, 256) == 512
    assert tier(255, 512, 256) == 512
    assert tier(300, 512, 256) == 1024  # 212 pairs of slack < 256: one more step
    assert tier(511, 512, 256) == 1024
    assert tier(512, 512, 256) == 1024  # strictly above the demand
    assert tier(1027, 512, 0) == 1536
    assert tier(1027, 32, 32) == 1088


def test_smallest_fitting_key():
    assert smallest_fitting_key([1024, 1536, 2048], 1000, 512) == 1024
    assert smallest_fitting_key([1024, 1536], 1024, 512) == 1536  # a bucket must exceed the demand
    assert smallest_fitting_key([1024], 1200, 512) is None
    assert smallest_fitting_key([], 10, 512) is None


def test_select_capture_replay_rebind():
    r = BucketedGraphRunner(model=None)
    assert r.select(135, 1027) == (tier(1027, 512, 256), "capture")
    r.cache, r._n_real = {1536: {}}, 135
    assert r.select(135, 1027) == (1536, None)
    assert r.select(135, 900) == (1536, None)  # a larger cached bucket is reused
    assert r.select(135, 1400) == (1536, None)
    assert r.select(135, 1536) == (tier(1536, 512, 256), "capture")  # no cached bucket above the demand
    assert r.select(136, 900)[1] == "rebind"


def test_arguments():
    with pytest.raises(ValueError):
        BucketedGraphRunner(model=None, task="efs")
    with pytest.raises(ValueError):
        BucketedGraphRunner(model=None, u_step=0)
