"""Drop-in replacement of the reference's plattice.py (plattice.py:7-23).

``PermutoLatticeFunction`` is the autograd Function: forward returns the
filtered values and saves ``(weight, feature)``; backward returns
``(None, grad_values)``: no gradient flows to the features, as in the
reference (plattice.py:19).  ``PermutoLattice`` is the nn.Module wrapper.

Unlike the reference, the lattice that forward builds is kept on the autograd
context and reused by backward (no rebuild).
"""
import torch
from torch.autograd import Function
from torch.autograd.function import once_differentiable
from torch.nn import Module

from . import PLOO

__all__ = ["PermutoLatticeFunction", "PermutoLattice"]


class PermutoLatticeFunction(Function):
    @staticmethod
    def forward(ctx, feature, values):
        weight, out, lat = PLOO.lattice_forward(feature, values)
        ctx.save_for_backward(weight, feature)
        ctx.lattice = lat
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
