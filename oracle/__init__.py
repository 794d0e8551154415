"""CPU oracle for the permutohedral-lattice filter (numpy front end).

TEST INFRASTRUCTURE ONLY: imported by tests/, by the smoke check and by the
CPU-baseline leg of bench.py, always as the checker and never as the thing
measured or shipped.  The product (plattice_pytorch_b200) never imports it.

The arithmetic lives in plattice_oracle.c (a sequential restatement of the
reference's permutohedral.cu, cited there line by line); this module loads it
with ctypes and wraps it for numpy arrays.  ``ref`` (oracle/ref.py) wraps the
reference CUDA filter built from its own sources into oracle/_ref/.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libplattice_oracle.so")

# Contraction variant of the reference build's float steps (bit mask, see
# plattice_oracle.c).  Pinned against the reference's own outputs: the golden
# vectors in tests/golden were produced by the reference CUDA build and the
# oracle reproduces their per-slot keys and weights exactly with this value.
ELEV_FMA_SUB, ELEV_FMA_ADD, BARY_FMA, SLICE_FMA = 1, 2, 4, 8
DEFAULT_VARIANT = ELEV_FMA_SUB | ELEV_FMA_ADD | BARY_FMA | SLICE_FMA

_lib = None


def build():
    """Compile plattice_oracle.c into libplattice_oracle.so (gcc)."""
    subprocess.run(["make", "-s", "-C", HERE, "libplattice_oracle.so"], check=True)


def lib():
    global _lib
    if _lib is None:
        src = os.path.join(HERE, "plattice_oracle.c")
        if (not os.path.exists(LIB_PATH)
                or os.path.getmtime(LIB_PATH) < os.path.getmtime(src)):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P, I, Lg = ctypes.c_void_p, ctypes.c_int, ctypes.c_long
        L.po_embed_all.argtypes = [P, Lg, I, I, P, P]
        L.po_embed_all.restype = I
        L.po_vertex_keys.argtypes = [P, Lg, I, I, P, Lg, P]
        L.po_vertex_keys.restype = Lg
        L.po_forward.argtypes = [P, P, Lg, I, I, I, P, P]
        L.po_forward.restype = Lg
        L.po_backward.argtypes = [P, P, P, Lg, I, I, I, P]
        L.po_backward.restype = Lg
        L.po_feature_grad.argtypes = [P, P, P, Lg, I, I, I, P]
        L.po_feature_grad.restype = Lg
        L.po_brute_gaussian.argtypes = [P, P, P, Lg, I, I, Lg, Lg, I, I, P]
        L.po_brute_gaussian.restype = I
        L.po_scale_factors_out.argtypes = [I, P]
        L.po_scale_factors_out.restype = None
        _lib = L
    return _lib


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _dims(features):
    f = _f32(features)
    pd = f.shape[-1]
    n = f.size // pd
    return f, n, pd


def scale_factors(pd):
    sf = np.zeros(pd, np.float32)
    lib().po_scale_factors_out(pd, _ptr(sf))
    return sf


def embed(features, variant=DEFAULT_VARIANT):
    """Per-slot lattice keys ``[n, pd+1, pd]`` int16 and barycentric weights
    ``[n, pd+1]`` float32 for every pixel (no hashing)."""
    f, n, pd = _dims(features)
    keys = np.zeros((n, pd + 1, pd), np.int16)
    w = np.zeros((n, pd + 1), np.float32)
    rc = lib().po_embed_all(_ptr(f), n, pd, variant, _ptr(keys), _ptr(w))
    if rc != 0:
        raise ValueError(f"po_embed_all failed with status {rc}")
    return keys, w


def vertex_keys(features, variant=DEFAULT_VARIANT):
    """Distinct lattice vertex keys ``[m, pd]`` int16 (first-seen order) and the
    per-slot vertex ids ``[n, pd+1]`` int32."""
    f, n, pd = _dims(features)
    cap = n * (pd + 1)
    keys = np.zeros((cap, pd), np.int16)
    sv = np.zeros((n, pd + 1), np.int32)
    m = lib().po_vertex_keys(_ptr(f), n, pd, variant, _ptr(keys), cap, _ptr(sv))
    if m < 0:
        raise ValueError(f"po_vertex_keys failed with status {-m}")
    return keys[:m].copy(), sv


def forward(features, values, variant=DEFAULT_VARIANT):
    """Return ``(weight [..., 1], out [..., vd], m)`` like the reference's forward."""
    f, n, pd = _dims(features)
    v = _f32(values)
    vd = v.shape[-1]
    out = np.zeros(v.shape, np.float32)
    wo = np.zeros(v.shape[:-1] + (1,), np.float32)
    m = lib().po_forward(_ptr(f), _ptr(v), n, pd, vd, variant, _ptr(out), _ptr(wo))
    if m < 0:
        raise ValueError(f"po_forward failed with status {-m}")
    return wo, out, int(m)


def feature_grad(features, values, grad, variant=DEFAULT_VARIANT):
    """Gradient ``[..., pd]`` of ``sum(grad * forward(features, values).out)``
    with respect to the features (the reference provides none); see
    po_feature_grad in plattice_oracle.c."""
    f, n, pd = _dims(features)
    v = _f32(values)
    g = _f32(grad)
    vd = v.shape[-1]
    out = np.zeros(f.shape, np.float32)
    m = lib().po_feature_grad(_ptr(f), _ptr(v), _ptr(g), n, pd, vd, variant, _ptr(out))
    if m < 0:
        raise ValueError(f"po_feature_grad failed with status {-m}")
    return out.reshape(np.shape(features))


def backward(features, grad, weight, variant=DEFAULT_VARIANT):
    """Value gradient like the reference's backward(features, grad, weight)."""
    f, n, pd = _dims(features)
    g = _f32(grad)
    wt = _f32(weight)
    vd = g.shape[-1]
    out = np.zeros(g.shape, np.float32)
    m = lib().po_backward(_ptr(f), _ptr(g), _ptr(wt), n, pd, vd, variant, _ptr(out))
    if m < 0:
        raise ValueError(f"po_backward failed with status {-m}")
    return out


def brute_gaussian(features, values, rows=None, threads=1, weight=None):
    """Exact dense Gaussian filter out_p = sum_q g_pq v_q / sum_q g_pq with
    g_pq = exp(-|f_p - f_q|^2 / 2), for flat output pixels ``rows`` (a range;
    default all).  With ``weight`` given it computes the value gradient
    sum_q g_pq weight_q v_q instead (values = upstream gradient).  float64."""
    f, n, pd = _dims(features)
    v = _f32(values).reshape(n, -1)
    vd = v.shape[1]
    p0, p1 = (0, n) if rows is None else (rows.start, rows.stop)
    out = np.zeros((p1 - p0, vd), np.float64)
    wt = None if weight is None else _f32(weight).reshape(n)
    rc = lib().po_brute_gaussian(_ptr(f), _ptr(v), None if wt is None else _ptr(wt), n, pd, vd,
                                 p0, p1, 0 if wt is None else 1, threads, _ptr(out))
    if rc != 0:
        raise ValueError(f"po_brute_gaussian failed with status {rc}")
    return out
