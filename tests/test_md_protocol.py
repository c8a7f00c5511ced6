"""Restart files and extxyz frames (fastmd/execution/md_protocol.py:93-201): the reference's restart
layout and format tag, atomic writes, continuation checks; frames read back. No device work."""
import json

import numpy as np
import pytest

from fastmd_b200.md_protocol import (RESTART_FORMAT, ExtxyzTrajectory, RestartData, read_extxyz, read_restart,
                                     resume_mismatch, write_restart)


def _data(n=5, nhc=True):
    rng = np.random.default_rng(0)
    return RestartData(ids=np.arange(n), numbers=np.array([55, 50, 53, 53, 53][:n]), masses=rng.random(n) + 1,
                       positions=rng.random((n, 3)), momenta=rng.standard_normal((n, 3)),
                       forces=rng.standard_normal((n, 3)).astype(np.float32), energy=np.array([-12.5]),
                       reference_energy=np.array([-3.25]), cell=np.eye(3) * 6.2, pbc=np.ones(3, bool), step=40,
                       parameters={"ensemble": "nvt_nhc" if nhc else "nve", "tchain": 3, "timestep": 0.1},
                       temperature_K=500.0 if nhc else None,
                       nhc_state={"eta": np.arange(3.0), "p_eta": -np.arange(3.0), "temperature_K": 500.0} if nhc
                       else None, offsets={"trajectory.extxyz": 1234}, engine="native")


@pytest.mark.parametrize("nhc", [True, False])
def test_restart_round_trip(tmp_path, nhc):
    d = _data(nhc=nhc)
    path = tmp_path / "restart.npz"
    write_restart(path, d)
    assert not any(p.name.endswith(".tmp.npz") for p in tmp_path.iterdir())  # atomic: no temporary left
    with np.load(path) as raw:  # the reference's field names and tag
        assert str(raw["format"]) == RESTART_FORMAT == "fastmd.distributed.md/1"
        assert {"ids", "numbers", "masses", "positions", "momenta", "forces", "potential_energy",
                "reference_energy", "cell", "pbc", "step", "parameters", "temperature_K", "nhc_eta", "nhc_p_eta",
                "offsets", "engine"} == set(raw.files) - {"format"}
        assert json.loads(str(raw["offsets"])) == d.offsets
    r = read_restart(path)
    for k in ("ids", "numbers", "masses", "positions", "momenta", "forces", "energy", "reference_energy", "cell",
              "pbc"):
        np.testing.assert_array_equal(getattr(r, k), getattr(d, k))
    assert (r.step, r.parameters, r.temperature_K, r.offsets, r.engine) == (
        d.step, d.parameters, d.temperature_K, d.offsets, d.engine)
    if nhc:
        np.testing.assert_array_equal(r.nhc_state["eta"], d.nhc_state["eta"])
        np.testing.assert_array_equal(r.nhc_state["p_eta"], d.nhc_state["p_eta"])
    else:
        assert r.nhc_state is None


def test_foreign_file_and_missing_engine(tmp_path):
    np.savez(tmp_path / "x.npz", format=np.array("something/else"))
    with pytest.raises(ValueError):
        read_restart(tmp_path / "x.npz")
    d = _data()
    write_restart(tmp_path / "r.npz", d)
    with np.load(tmp_path / "r.npz") as raw:
        fields = {k: raw[k] for k in raw.files if k != "engine"}
    np.savez(tmp_path / "old.npz", **fields)
    assert read_restart(tmp_path / "old.npz").engine == "domain"


def test_resume_mismatch():
    saved = {"timestep": 0.1, "tchain": 3, "total_steps": 100, "ramp": None}
    assert resume_mismatch(saved, dict(saved, total_steps=500)) == {}
    assert resume_mismatch(saved, dict(saved, tchain=4)) == {"tchain": (3, 4)}
    assert resume_mismatch(saved, {**saved, "extra": 1}) == {"extra": (None, 1)}
    assert resume_mismatch(saved, dict(saved, tchain=4), ignore=("tchain",)) == {}


def test_extxyz_frames_round_trip(tmp_path):
    rng = np.random.default_rng(1)
    path = tmp_path / "traj.extxyz"
    traj = ExtxyzTrajectory(path)
    frames = []
    for step in (0, 10):
        f = dict(numbers=np.array([55, 50, 53]), positions=rng.random((3, 3)) * 6, cell=np.diag([6.2, 6.3, 6.4]),
                 pbc=np.array([True, True, False]), velocities=rng.standard_normal((3, 3)),
                 forces=rng.standard_normal((3, 3)), energy=-7.125 - step, info={"step": np.int64(step),
                                                                                 "temperature": 500.5})
        traj.write(**f)
        frames.append(f)
        assert traj.tell() == path.stat().st_size  # flushed: the size is a frame boundary
    traj.close()
    ExtxyzTrajectory(path, append=True).close()
    back = read_extxyz(path)
    assert len(back) == 2
    for f, b in zip(frames, back):
        np.testing.assert_array_equal(b["numbers"], f["numbers"])
        for k in ("positions", "velocities", "forces"):
            np.testing.assert_allclose(b[k], f[k], atol=1e-8)
        np.testing.assert_array_equal(b["cell"], f["cell"])
        np.testing.assert_array_equal(b["pbc"], f["pbc"])
        assert b["energy"] == f["energy"] and b["step"] == int(f["info"]["step"]) and b["temperature"] == 500.5
    with pytest.raises(ValueError):
        ExtxyzTrajectory(tmp_path / "t2.extxyz").write(numbers=[1], positions=np.zeros((1, 3)), cell=np.eye(3),
                                                      pbc=[1, 1, 1], velocities=np.zeros((1, 3)),
                                                      forces=np.zeros((1, 3)), energy=0.0, info={"v": [1, 2]})
