"""ASE's unit system (eV, Angstrom, amu) from the CODATA 2014 constants -- test oracle.

ASE 3.29 derives its units from CODATA 2014 (its default ``CODATA`` version):
kB = k / e (eV/K), the ASE time unit is Angstrom * sqrt(amu / eV), so one
second is 1e10 * sqrt(e / amu) ASE time units. ASE itself is absent from this
container; the values below are the published constants and those
definitions (the one unpinned input of the NHC oracle, shared bit for bit by
the product, which takes the same Python floats).
"""
import math

_e = 1.6021766208e-19      # C (CODATA 2014)
_amu = 1.660539040e-27     # kg (CODATA 2014)
_k = 1.38064852e-23        # J/K (CODATA 2014)

kB = _k / _e
second = 1e10 * math.sqrt(_e / _amu)
fs = 1e-15 * second
Pascal = (1 / _e) / 1e30
GPa = 1e9 * Pascal
