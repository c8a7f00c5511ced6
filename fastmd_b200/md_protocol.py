"""Restart files and trajectory frames of the GPU-resident MD (fastmd/execution/md_protocol.py).

``RestartData`` / ``write_restart`` / ``read_restart`` / ``resume_mismatch`` keep the reference's restart
file (md_protocol.py:123-201): one ``.npz`` per state, tagged ``"fastmd.distributed.md/1"``, rows in ID
order, the cached evaluation of the state (a continuation does not re-evaluate), the NHC chain, the
driver's parameters and the output files' sizes, written atomically (temporary file, then rename), so a
file written here continues under the reference and the other way round. ``ExtxyzTrajectory``
(md_protocol.py:93) writes extended-XYZ frames with velocities instead of momenta, the energy, forces and
the scalar extras of each frame in the comment line, flushed per frame so the file size is a frame
boundary (the offset a restart records); it needs no ASE: the comment line and columns are written here
in the extxyz layout (``Lattice``, ``Properties=species:S:1:pos:R:3:velocities:R:3:forces:R:3``,
``pbc``), and ``read_extxyz`` reads them back.
"""
from __future__ import annotations

import json
import math
import os
from dataclasses import dataclass
from pathlib import Path

import numpy as np

RESTART_FORMAT = "fastmd.distributed.md/1"

_SYMBOLS = ("X H He Li Be B C N O F Ne Na Mg Al Si P S Cl Ar K Ca Sc Ti V Cr Mn Fe Co Ni Cu Zn Ga Ge As Se Br Kr "
            "Rb Sr Y Zr Nb Mo Tc Ru Rh Pd Ag Cd In Sn Sb Te I Xe Cs Ba La Ce Pr Nd Pm Sm Eu Gd Tb Dy Ho Er Tm Yb "
            "Lu Hf Ta W Re Os Ir Pt Au Hg Tl Pb Bi Po At Rn Fr Ra Ac Th Pa U Np Pu Am Cm Bk Cf Es Fm Md No Lr").split()


@dataclass
class RestartData:
    """One restart file as host arrays, rows in ID order (md_protocol.py:123): ``ids``/``numbers`` int64,
    ``masses``, ``positions`` (float64 for nvt_nhc) and ``momenta`` float64, the cached ``forces``
    (float32), ``energy`` and ``reference_energy``, ``cell``, ``pbc``, ``step``, the driver's
    ``parameters``, the thermostat target ``temperature_K`` (None for nve), ``nhc_state`` (``eta``,
    ``p_eta``, ``temperature_K``; None unless nvt_nhc), the output files' ``offsets`` and the writing
    ``engine``."""

    ids: np.ndarray
    numbers: np.ndarray
    masses: np.ndarray
    positions: np.ndarray
    momenta: np.ndarray
    forces: np.ndarray
    energy: np.ndarray
    reference_energy: np.ndarray
    cell: np.ndarray
    pbc: np.ndarray
    step: int
    parameters: dict
    temperature_K: float | None
    nhc_state: dict | None
    offsets: dict
    engine: str


def write_restart(path, data: RestartData) -> None:
    """Write ``data`` atomically (a temporary ``.npz`` next to ``path``, then ``os.replace``)."""
    path = Path(path)
    nhc = {} if data.nhc_state is None else data.nhc_state
    temporary = path.with_name(path.name + ".tmp.npz")
    np.savez(temporary, format=np.array(RESTART_FORMAT), ids=np.asarray(data.ids, np.int64),
             numbers=np.asarray(data.numbers, np.int64), masses=np.asarray(data.masses, np.float64),
             positions=np.asarray(data.positions), momenta=np.asarray(data.momenta, np.float64),
             forces=np.asarray(data.forces), potential_energy=np.asarray(data.energy),
             reference_energy=np.asarray(data.reference_energy), cell=np.asarray(data.cell),
             pbc=np.asarray(data.pbc), step=np.array(int(data.step), dtype=np.int64),
             parameters=np.array(json.dumps(data.parameters)),
             temperature_K=np.array(math.nan if data.temperature_K is None else float(data.temperature_K)),
             nhc_eta=np.asarray(nhc.get("eta", np.zeros(0)), np.float64),
             nhc_p_eta=np.asarray(nhc.get("p_eta", np.zeros(0)), np.float64),
             offsets=np.array(json.dumps(data.offsets)), engine=np.array(data.engine))
    os.replace(temporary, path)


def read_restart(path) -> RestartData:
    """Parse a restart file (format tag checked; a file without ``engine`` reads as "domain")."""
    with np.load(path) as data:
        if str(data["format"]) != RESTART_FORMAT:
            raise ValueError(f"not a {RESTART_FORMAT} restart file")
        parameters = json.loads(str(data["parameters"]))
        temperature = float(data["temperature_K"])
        nhc = parameters.get("ensemble") == "nvt_nhc"
        return RestartData(
            ids=data["ids"], numbers=data["numbers"], masses=data["masses"], positions=data["positions"],
            momenta=data["momenta"], forces=data["forces"], energy=data["potential_energy"],
            reference_energy=data["reference_energy"], cell=data["cell"], pbc=data["pbc"], step=int(data["step"]),
            parameters=parameters, temperature_K=None if math.isnan(temperature) else temperature,
            nhc_state={"temperature_K": temperature, "eta": np.array(data["nhc_eta"]),
                       "p_eta": np.array(data["nhc_p_eta"])} if nhc else None,
            offsets=json.loads(str(data["offsets"])),
            engine=str(data["engine"]) if "engine" in data.files else "domain")


def resume_mismatch(saved: dict, requested: dict, *, ignore=()) -> dict:
    """``{key: (saved, requested)}`` for every parameter a continuation changes, keys sorted;
    ``total_steps`` and the keys in ``ignore`` never count (md_protocol.py:193)."""
    skip = {"total_steps", *ignore}
    return {key: (saved.get(key), requested.get(key)) for key in sorted(saved.keys() | requested.keys())
            if key not in skip and saved.get(key) != requested.get(key)}


def _fmt(value) -> str:
    if isinstance(value, (bool, np.bool_)):
        return "T" if value else "F"
    if isinstance(value, (int, np.integer)):
        return str(int(value))
    return repr(float(value))


class ExtxyzTrajectory:
    """Truncatable extended-XYZ trajectory (md_protocol.py:93): one flushed frame per ``write``."""

    def __init__(self, path, *, append: bool = False):
        self._stream = open(path, "a" if append else "w", encoding="utf-8")

    def write(self, *, numbers, positions, cell, pbc, velocities, forces, energy: float, info: dict | None = None):
        """One frame: ``velocities`` in Angstrom per ASE time unit (momenta / masses); ``info`` scalar
        extras (``step`` an integer)."""
        numbers = np.asarray(numbers).reshape(-1)
        pos, vel, frc = (np.asarray(a, np.float64).reshape(-1, 3) for a in (positions, velocities, forces))
        cell = np.asarray(cell, np.float64).reshape(3, 3)
        pbc = np.asarray(pbc, bool).reshape(3)
        extras = {"energy": float(energy)}
        for key, value in (info or {}).items():
            value = np.asarray(value)
            if value.size != 1:
                raise ValueError(f"frame extra {key!r} must be a scalar")
            extras[key] = int(value.item()) if key == "step" else float(value.item())
        comment = (f'Lattice="{" ".join(repr(float(v)) for v in cell.reshape(-1))}" '
                   "Properties=species:S:1:pos:R:3:velocities:R:3:forces:R:3 "
                   + " ".join(f"{k}={_fmt(v)}" for k, v in extras.items())
                   + f' pbc="{" ".join(_fmt(b) for b in pbc)}"')
        lines = [str(numbers.size), comment]
        for z, p, v, f in zip(numbers, pos, vel, frc):
            lines.append(f"{_SYMBOLS[int(z)]:<2} " + " ".join(f"{x:16.8f}" for x in (*p, *v, *f)))
        self._stream.write("\n".join(lines) + "\n")
        self._stream.flush()

    def tell(self) -> int:
        """The file size: a frame boundary after every write."""
        return self._stream.tell()

    def close(self) -> None:
        self._stream.close()


def read_extxyz(path) -> list[dict]:
    """The frames of an ``ExtxyzTrajectory`` file: numbers, positions, velocities, forces, cell, pbc and
    the comment line's scalars."""
    frames = []
    with open(path, encoding="utf-8") as f:
        lines = f.read().splitlines()
    i = 0
    while i < len(lines):
        n = int(lines[i])
        comment = lines[i + 1]
        fields, key, buf, quoted = {}, "", "", False
        for token in comment.replace('"', ' " ').split():
            if token == '"':
                quoted = not quoted
                if not quoted:
                    fields[key] = buf.strip()
                continue
            if quoted:
                buf += " " + token
            elif "=" in token:
                key, value = token.split("=", 1)
                if value:
                    fields[key] = value
                else:
                    buf = ""
        rows = [line.split() for line in lines[i + 2:i + 2 + n]]
        data = np.array([[float(x) for x in row[1:]] for row in rows])
        frame = {"numbers": np.array([_SYMBOLS.index(row[0]) for row in rows]), "positions": data[:, 0:3],
                 "velocities": data[:, 3:6], "forces": data[:, 6:9],
                 "cell": np.array([float(v) for v in fields.pop("Lattice").split()]).reshape(3, 3),
                 "pbc": np.array([v == "T" for v in fields.pop("pbc").split()])}
        fields.pop("Properties")
        for k, v in fields.items():
            frame[k] = int(v) if k == "step" else float(v)
        frames.append(frame)
        i += 2 + n
    return frames


__all__ = ["ExtxyzTrajectory", "RESTART_FORMAT", "RestartData", "read_extxyz", "read_restart", "resume_mismatch",
           "write_restart"]
