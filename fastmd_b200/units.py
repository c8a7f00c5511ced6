"""ASE's unit system (eV, Angstrom, amu, ASE time) from the CODATA 2014 constants.

ASE 3.29, which the reference integrator ports (fastmd/execution/gpu_nhc.py:1),
derives kB = k / e (eV/K) and its time unit Angstrom * sqrt(amu / eV), i.e. one
second is 1e10 * sqrt(e / amu) ASE time units. The same expressions give the
same floats, so thermostat constants formed here equal ASE's bit for bit.
"""
import math

_e = 1.6021766208e-19      # elementary charge, C (CODATA 2014)
_amu = 1.660539040e-27     # atomic mass unit, kg (CODATA 2014)
_k = 1.38064852e-23        # Boltzmann constant, J/K (CODATA 2014)

kB = _k / _e
second = 1e10 * math.sqrt(_e / _amu)
fs = 1e-15 * second
Pascal = (1 / _e) / 1e30
GPa = 1e9 * Pascal
