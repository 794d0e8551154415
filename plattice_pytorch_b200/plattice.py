"""Drop-in replacement of the reference's plattice.py (plattice.py:7-23).

``PermutoLatticeFunction`` is the autograd Function: forward returns the
filtered values and saves ``(weight, feature)``; backward returns
``(None, grad_values)``: no gradient flows to the features, as in the
reference (plattice.py:19).  ``PermutoLattice`` is the nn.Module wrapper.

Unlike the reference, the lattice that forward builds is kept on the autograd
context and reused by backward (no rebuild), unless ``PLOO.set_keep_lattice(False)``
(or PLATTICE_KEEP_LATTICE=0) asks for the reference's behaviour: nothing kept,
the lattice rebuilt in backward.

``PermutoLatticeBatchFunction`` (no counterpart in the reference) is
``PermutoLatticeFunction`` over a batch ``[B,H,W,...]`` in one library call,
one lattice per image.

``PermutoLatticeFeatureFunction`` (no counterpart in the reference) is
``PermutoLatticeFunction`` with a gradient for the features as well: the
slope of the piecewise-linear filter inside each pixel's simplex.

``LatticeFilterFunction`` (no counterpart in the reference) filters further
values on a kept lattice -- the ``PLOO.Lattice`` of an earlier forward on the
same features -- without rebuilding it, as the iterations of a mean-field CRF
do; its backward is the value gradient on the same lattice.
"""
import ctypes

import torch
from torch.autograd import Function
from torch.autograd.function import once_differentiable
from torch.nn import Module

from . import PLOO, _lib

_UNSET = object()
_EXT = _UNSET


def _cpp_function():
    """The C++ build of PermutoLatticeFunction (extension module _plattice_torch,
    built next to the library), pointed at the loaded library's entry points;
    None when the extension is not built."""
    global _EXT
    if _EXT is _UNSET:
        try:
            from . import _plattice_torch as m
        except ImportError:
            _EXT = None
            return None
        L = _lib.lib()
        addr = lambda f: ctypes.cast(f, ctypes.c_void_p).value
        m.set_entry_points(addr(L.plattice_forward), addr(L.plattice_backward), addr(L.plattice_workspace_sizes),
                           addr(L.plattice_reuse_scratch_size), addr(L.plattice_error_string),
                           addr(L.plattice_last_error_detail))
        _EXT = m.permuto_lattice
    return _EXT

__all__ = ["PermutoLatticeFunction", "PermutoLattice", "LatticeFilterFunction", "PermutoLatticeBatchFunction",
           "PermutoLatticeFeatureFunction"]


class PermutoLatticeFunction(Function):
    """``PermutoLatticeFunction.apply(feature, values) -> out``.

    ``apply`` runs the C++ build of this Function (the same checks, messages,
    kept lattice and library calls as forward / backward below, without the
    Python interpreter between the autograd engine and the library) when the
    extension is built and PLATTICE_CHECK is off; otherwise, and for arguments
    that are not tensors, the Python Function below.  Either way the filter
    runs in libplattice_b200.so."""

    @classmethod
    def apply(cls, feature, values):
        fn = None if PLOO._CHECK else _cpp_function()
        if fn is not None and type(feature) is torch.Tensor and type(values) is torch.Tensor:
            return fn(feature, values, PLOO._KEEP)
        return super().apply(feature, values)

    @staticmethod
    def forward(ctx, feature, values):
        weight, out, lat = PLOO.lattice_forward(feature, values)
        ctx.save_for_backward(weight, feature)
        ctx.lattice = lat if PLOO._KEEP else None
        return out

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_output):
        weight, feature = ctx.saved_tensors
        grad_values = PLOO.lattice_backward(feature, grad_output.contiguous(), weight,
                                            getattr(ctx, "lattice", None), saved=True)
        return None, grad_values


class PermutoLattice(Module):
    def forward(self, feature, values):
        return PermutoLatticeFunction.apply(feature, values)


class LatticeFilterFunction(Function):
    """``LatticeFilterFunction.apply(values, lattice) -> out``: the forward filter
    of ``values`` on the kept ``lattice``; gradient to ``values`` only."""

    @staticmethod
    def forward(ctx, values, lattice):
        weight, out = PLOO.lattice_filter(lattice, values)
        ctx.save_for_backward(weight)
        ctx.lattice = lattice
        return out

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_output):
        (weight,) = ctx.saved_tensors
        return PLOO.lattice_filter_backward(ctx.lattice, grad_output.contiguous(), weight), None


class PermutoLatticeBatchFunction(Function):
    """``PermutoLatticeBatchFunction.apply(features [B,H,W,pd], values [B,H,W,vd])``."""

    @staticmethod
    def forward(ctx, feature, values):
        weight, out, lat = PLOO.batch_forward(feature, values)
        ctx.save_for_backward(weight, feature)
        ctx.lattice = lat if PLOO._KEEP else None
        return out

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_output):
        weight, feature = ctx.saved_tensors
        grad_values = PLOO.batch_backward(feature, grad_output.contiguous(), weight,
                                          getattr(ctx, "lattice", None), saved=True)
        return None, grad_values


class PermutoLatticeFeatureFunction(Function):
    """``PermutoLatticeFeatureFunction.apply(features, values) -> out`` with
    gradients for both inputs."""

    @staticmethod
    def forward(ctx, feature, values):
        weight, out, lat = PLOO.lattice_forward(feature, values)
        ctx.save_for_backward(weight, feature, values, out)
        ctx.lattice = lat
        return out

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_output):
        weight, feature, values, out = ctx.saved_tensors
        g = grad_output.contiguous()
        grad_features = None
        if ctx.needs_input_grad[0]:
            grad_features = PLOO.feature_grad(ctx.lattice, feature, values, g, weight, out)
        grad_values = None
        if ctx.needs_input_grad[1]:
            grad_values = PLOO.lattice_backward(feature, g, weight, ctx.lattice, saved=True)
        return grad_features, grad_values
