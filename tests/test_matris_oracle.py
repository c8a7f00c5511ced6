"""The FP64 MatRIS oracle against the reference's own MatRIS-10M (tests/golden/matris.npz, made by running
fastmd/models/matris/model.py:99 on CPU in float64 and float32 with the seeded weights of
``fastmd_b200.matris_params.seeded_parameters``): the oracle's energy, forces and stress agree with the
reference's float64 evaluation to 1e-10 relative."""
import numpy as np
import pytest

from conftest import golden
from fastmd_b200.matris_params import MATRIS_10M, parameter_shapes, seeded_parameters
from oracle import matris as om


def _case(g, seed, positions_key):
    t = f"matris_s{seed}"
    return dict(positions=g[f"{t}_{positions_key}"].astype(np.float64), cell=g[f"{t}_cell"],
                numbers=g[f"{t}_numbers"], edge_index=g[f"{t}_edge_index"], edge_image=g[f"{t}_edge_image"],
                d2u=g[f"{t}_d2u"], u2d=g[f"{t}_u2d"], line_graph=g[f"{t}_line_graph"])


def test_seeded_parameters_match_the_fixture():
    g = golden("matris")
    params = seeded_parameters(MATRIS_10M, seed=0)
    assert set(params) == {k for k, _, _ in parameter_shapes(MATRIS_10M)}
    total = sum(float(v.astype(np.float64).sum()) for v in params.values())
    assert total == float(g["matris_param_sum"])
    assert sum(v.size for v in params.values()) == 10_459_923  # MatRIS-10M with energy head (256, 256)


@pytest.mark.parametrize("seed", [0, 1])
def test_oracle_equals_reference_float64(seed):
    g = golden("matris")
    t = f"matris_s{seed}"
    e, f, s = om.energy_forces_stress(seeded_parameters(MATRIS_10M, 0), MATRIS_10M, **_case(g, seed, "positions64"))
    assert abs(e - float(g[f"{t}_e64"])) <= 1e-10 * abs(e)
    assert np.abs(f - g[f"{t}_f64"]).max() <= 1e-10 * np.abs(f).max()
    assert np.abs(s - g[f"{t}_s64"]).max() <= 1e-10 * np.abs(s).max()
    # the reference's own float32 evaluation sits within its FP32 rounding of the same result
    e32, f32, s32 = om.energy_forces_stress(seeded_parameters(MATRIS_10M, 0), MATRIS_10M,
                                            **_case(g, seed, "positions"))
    assert abs(float(g[f"{t}_e32"]) - e32) <= 1e-6 * abs(e32)
    assert np.abs(g[f"{t}_f32"] - f32).max() <= 1e-4 * np.abs(f32).max()
    assert np.abs(g[f"{t}_s32"] - s32).max() <= 1e-5 * np.abs(s32).max()


def test_graph_counts():
    g = golden("matris")
    for seed in (0, 1):
        t = f"matris_s{seed}"
        assert g[f"{t}_edge_index"].shape[0] == 2 * g[f"{t}_u2d"].shape[0] > 2000  # about 2,054 directed edges
        assert g[f"{t}_line_graph"].shape[1] == 5 and g[f"{t}_line_graph"].shape[0] > 17_000


def test_config_from_a_reference_checkpoint_config():
    from fastmd_b200.matris_params import MatRISConfig

    ref = MATRIS_10M.reference_kwargs()
    assert MatRISConfig.from_reference(ref) == MATRIS_10M
    with pytest.raises(NotImplementedError):
        MatRISConfig.from_reference({**ref, "norm_type": "rms"})
    with pytest.raises(NotImplementedError):
        MatRISConfig.from_reference({**ref, "three_body_expansion": "SH"})
