"""The reference CUDA filter, built from its own sources into oracle/_ref/.

TEST INFRASTRUCTURE ONLY (tests, golden-vector script, reference arm of the
benchmark).  Needs a GPU and the prebuilt files from ``make -C oracle ref``.

* :class:`RefLattice` calls the reference entry points permuto_filter /
  permuto_filter_grad (permutohedral.cu:685,717) through oracle/ref_harness.cu
  with caller-owned workspace, so that the lattice the reference built (its
  per-slot matrix and hash-table keys) can be read back: canonical slots are
  those whose matrix index points to themselves (the test the reference itself
  uses, permutohedral.cu:332,357), their keys are the vertex key set.
* :func:`load_ploo` imports the reference's own torch extension (permuto.cpp),
  the reference's public API ``forward(features, values) -> [weight, out]`` /
  ``backward(features, grad, weight) -> grad_values``.
"""
import ctypes
import importlib.machinery
import importlib.util
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
REF_LIB = os.path.join(REF_DIR, "libplattice_ref.so")
PLOO_DIR = os.path.join(REF_DIR, "ploo")


def available():
    return os.path.exists(REF_LIB)


def ploo_available():
    return os.path.exists(os.path.join(PLOO_DIR, "PLOO_ref.so"))


_ploo = None


def load_ploo():
    """Import the reference torch extension module (PLOO_ref)."""
    global _ploo
    if _ploo is None:
        import torch  # noqa: F401  (the extension links against libtorch)
        path = os.path.join(PLOO_DIR, "PLOO_ref.so")
        loader = importlib.machinery.ExtensionFileLoader("PLOO_ref", path)
        spec = importlib.util.spec_from_file_location("PLOO_ref", path, loader=loader)
        mod = importlib.util.module_from_spec(spec)
        loader.exec_module(mod)
        _ploo = mod
    return _ploo


class RefLattice:
    """ctypes wrapper over libplattice_ref.so operating on torch CUDA tensors."""

    def __init__(self):
        import torch
        self.torch = torch
        L = ctypes.CDLL(REF_LIB)
        P, I = ctypes.c_void_p, ctypes.c_int
        L.ref_workspace_sizes.argtypes = [ctypes.c_longlong, I, I, ctypes.POINTER(ctypes.c_longlong)]
        L.ref_workspace_sizes.restype = None
        L.ref_forward.argtypes = [P] * 10 + [I] * 5
        L.ref_forward.restype = I
        L.ref_backward.argtypes = [P] * 10 + [I] * 5
        L.ref_backward.restype = I
        self.L = L

    def workspace(self, n, pd, vd, device):
        torch = self.torch
        sizes = (ctypes.c_longlong * 6)()
        self.L.ref_workspace_sizes(n, pd, vd, sizes)
        return [torch.empty(int(s), dtype=torch.uint8, device=device) for s in sizes]

    def _ptrs(self, ws):
        return [ctypes.c_void_p(t.data_ptr()) for t in ws]

    def forward(self, features, values, ws=None, sync=True):
        """Run the reference forward on CUDA tensors [H,W,pd], [H,W,vd];
        returns (weight [H,W,1], out [H,W,vd], workspace)."""
        torch = self.torch
        h, w, pd = features.shape
        vd = values.shape[2]
        if ws is None:
            ws = self.workspace(h * w, pd, vd, features.device)
        out = torch.empty((h, w, vd), dtype=torch.float32, device=features.device)
        wo = torch.zeros((h, w, 1), dtype=torch.float32, device=features.device)
        rc = self.L.ref_forward(ctypes.c_void_p(wo.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                ctypes.c_void_p(values.data_ptr()),
                                ctypes.c_void_p(features.data_ptr()), *self._ptrs(ws),
                                pd, vd, w, h, 1 if sync else 0)
        if rc != 0:
            raise RuntimeError(f"reference forward: CUDA error {rc}")
        return wo, out, ws

    def backward(self, features, grad, weight, ws=None, sync=True):
        torch = self.torch
        h, w, pd = features.shape
        vd = grad.shape[2]
        if ws is None:
            ws = self.workspace(h * w, pd, vd, features.device)
        out = torch.empty((h, w, vd), dtype=torch.float32, device=features.device)
        rc = self.L.ref_backward(ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(grad.data_ptr()),
                                 ctypes.c_void_p(weight.data_ptr()),
                                 ctypes.c_void_p(features.data_ptr()), *self._ptrs(ws),
                                 pd, vd, w, h, 1 if sync else 0)
        if rc != 0:
            raise RuntimeError(f"reference backward: CUDA error {rc}")
        return out

    @staticmethod
    def lattice(ws, n, pd):
        """Read back the lattice of the last call on ``ws``: per-slot keys
        [n,K,pd] int16, per-slot weights [n,K] float32, the sorted vertex key
        set [m,pd] int16 and m."""
        K = pd + 1
        mat = ws[0].cpu().numpy().view(np.int32).reshape(n * K, 2)
        idx = mat[:, 0].copy()
        wts = mat[:, 1].copy().view(np.float32).reshape(n, K)
        keys = ws[4].cpu().numpy().view(np.int16).reshape(n * K, pd)
        canon = np.nonzero(idx == np.arange(n * K))[0]
        slot_keys = keys[idx].reshape(n, K, pd)
        vkeys = sort_keys(keys[canon])
        return {"slot_keys": slot_keys, "slot_w": wts, "vertex_keys": vkeys, "m": int(canon.size)}


def sort_keys(keys):
    """Lexicographically sorted copy of an [m, pd] int16 key array."""
    keys = np.ascontiguousarray(keys, np.int16)
    if keys.shape[0] == 0:
        return keys
    order = np.lexsort(keys.T[::-1])
    return keys[order]
