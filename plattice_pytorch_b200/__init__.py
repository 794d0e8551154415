"""sm_100a permutohedral-lattice filter behind the reference's operator API.

``plattice_pytorch_b200.PLOO`` replaces the reference's ``PLOO`` extension
module (forward / backward) and ``plattice_pytorch_b200.plattice`` its
plattice.py (PermutoLatticeFunction, PermutoLattice).  The work is done by
libplattice_b200.so through the C ABI of include/plattice.h.
"""
from . import PLOO
from .plattice import (LatticeFilterFunction, PermutoLattice, PermutoLatticeBatchFunction,
                       PermutoLatticeFeatureFunction, PermutoLatticeFunction)

__all__ = ["PLOO", "PermutoLattice", "PermutoLatticeFunction", "PermutoLatticeBatchFunction",
           "PermutoLatticeFeatureFunction", "LatticeFilterFunction"]
