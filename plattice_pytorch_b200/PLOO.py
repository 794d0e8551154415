"""Drop-in replacement of the reference's extension module ``PLOO``.

The reference builds ``PLOO`` from permuto.cpp (setup.py:5-7) and calls it as
``PLOO.forward(features, values) -> [weight, out]`` and
``PLOO.backward(features, grad_values, weight) -> grad`` (permuto.cpp:71-158,
plattice.py:10,16).  This module keeps those names, argument meanings, return
order, input checks and error messages (permuto.cpp:33-40, 72-85, 113-132;
a failed check raises RuntimeError as TORCH_CHECK does) and runs the sm_100a
library through its C ABI (include/plattice.h).

Differences that a caller can observe only as speed:
  * ``backward`` reuses the lattice that ``forward`` built for the same
    ``features`` tensor (same object, unmodified since), instead of rebuilding
    it as permutohedral.cu:615-635 does; otherwise it rebuilds.
  * kernels run on PyTorch's current stream of the tensors' device, not on the
    legacy default stream, and no call synchronises the host.

Set the environment variable PLATTICE_CHECK=1 to synchronise after every call
and raise if the device reports a failure.
"""
import ctypes
import os
import weakref

import torch

from . import _lib

__all__ = ["forward", "backward", "Lattice", "lattice_forward", "lattice_backward",
           "lattice_filter", "lattice_filter_backward", "feature_grad", "BatchLattice", "batch_forward",
           "batch_backward", "forward_batch", "backward_batch", "lattice_info", "vertex_keys"]

_CHECK = os.environ.get("PLATTICE_CHECK", "0") not in ("", "0")


def _require(cond, msg):
    if not cond:
        raise RuntimeError(msg)


def _check_input(t, name):
    # CHECK_CUDA / CHECK_CONTIGUOUS of permuto.cpp:33-35
    _require(isinstance(t, torch.Tensor) and t.is_cuda, f"{name} must be CUDA")
    _require(t.is_contiguous(), f"{name} must be contiguous")


def _check_dims(pd, vd):
    # permuto.cpp:37-40
    _require(1 <= pd <= 16, "feature dimension pd must be in [1, 16]")
    _require(1 <= vd <= 8, "value dimension vd must be in [1, 8]")


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


class Lattice:
    """A lattice built on the device for one ``features`` tensor.

    Holds the lattice buffer (kept for backward calls), optionally the scratch
    buffer of the build (needed by :func:`vertex_keys`), and whether a
    backward pass has already used its value buffers."""

    __slots__ = ("buf", "scratch", "h", "w", "pd", "vd", "device", "used", "_feat_ref",
                 "_feat_version", "_feat_ptr", "__weakref__")

    def __init__(self, features, vd, buf, scratch):
        self.buf = buf
        self.scratch = scratch
        self.h, self.w, self.pd = (int(s) for s in features.shape)
        self.vd = int(vd)
        self.device = features.device
        self.used = False
        self._feat_ref = weakref.ref(features)
        self._feat_version = features._version
        self._feat_ptr = features.data_ptr()

    def matches(self, features, vd, same_object=True):
        """True when this lattice was built from ``features`` as it is now.
        ``same_object=False`` drops the identity test, for callers (autograd's
        saved tensors) that hand back a new tensor object over the same,
        version-checked storage."""
        if same_object and self._feat_ref() is not features:
            return False
        return (features.data_ptr() == self._feat_ptr and int(vd) == self.vd
                and tuple(features.shape) == (self.h, self.w, self.pd)
                and features.device == self.device
                and (not same_object or features._version == self._feat_version))


def _sync_check(lat, call):
    st = ctypes.c_int(0)
    rc = _lib.lib().plattice_lattice_info(_ptr(lat.buf), ctypes.byref(st), None, None, None,
                                          _stream(lat.device))
    if rc != _lib.OK:
        raise _lib.PlatticeError(call, rc, f"device status bits {st.value:#x}")


def lattice_forward(features, values, keep_scratch=False):
    """Forward filter; returns ``(weight [H,W,1], out [H,W,vd], Lattice)``."""
    _check_input(features, "features")
    _check_input(values, "values")
    _require(features.dim() == 3, "features must be [H, W, pd]")
    _require(values.dim() == 3, "values must be [H, W, vd]")
    _require(features.dtype == torch.float32, "features must be float32")
    _require(values.dtype == torch.float32, "values must be float32")
    _require(features.shape[0] == values.shape[0] and features.shape[1] == values.shape[1],
             "features and values must have matching H, W")
    h, w, pd = (int(s) for s in features.shape)
    vd = int(values.shape[2])
    _check_dims(pd, vd)
    _require(values.device == features.device, "features and values must be on the same device")
    dev = features.device
    with torch.cuda.device(dev):
        out = torch.empty((h, w, vd), dtype=torch.float32, device=dev)
        weight = torch.empty((h, w, 1), dtype=torch.float32, device=dev)
        lb, sb = _lib.workspace_sizes(h, w, pd, vd)
        buf = torch.empty(lb, dtype=torch.uint8, device=dev)
        scratch = torch.empty(sb, dtype=torch.uint8, device=dev)
        rc = _lib.lib().plattice_forward(_ptr(weight), _ptr(out), _ptr(values), _ptr(features),
                                         _ptr(buf), lb, _ptr(scratch), sb, pd, vd, w, h,
                                         _stream(dev))
        if rc != _lib.OK:
            raise _lib.PlatticeError("plattice_forward", rc, f"h={h} w={w} pd={pd} vd={vd}")
        lat = Lattice(features, vd, buf, scratch if keep_scratch else None)
        if _CHECK and h * w > 0:
            _sync_check(lat, "plattice_forward")
    return weight, out, lat


def lattice_backward(features, grad_values, weight_saved, lattice=None, saved=False):
    """Value gradient; reuses ``lattice`` when it was built from ``features``
    as they are now, else rebuilds.  ``saved=True`` when ``features`` comes
    from autograd's saved tensors (whose version check already guarantees
    they are unmodified).  Returns ``grad [H,W,vd]``."""
    _check_input(features, "features")
    _check_input(grad_values, "grad_values")
    _check_input(weight_saved, "weight_saved")
    _require(features.dim() == 3, "features must be [H, W, pd]")
    _require(grad_values.dim() == 3, "grad_values must be [H, W, vd]")
    _require(weight_saved.dim() == 3 and weight_saved.shape[2] == 1, "weight_saved must be [H, W, 1]")
    _require(features.dtype == torch.float32, "features must be float32")
    _require(grad_values.dtype == torch.float32, "grad_values must be float32")
    _require(weight_saved.dtype == torch.float32, "weight_saved must be float32")
    _require(features.shape[0] == grad_values.shape[0] and features.shape[1] == grad_values.shape[1],
             "features and grad_values must have matching H, W")
    _require(features.shape[0] == weight_saved.shape[0] and features.shape[1] == weight_saved.shape[1],
             "features and weight_saved must have matching H, W")
    h, w, pd = (int(s) for s in features.shape)
    vd = int(grad_values.shape[2])
    _check_dims(pd, vd)
    _require(grad_values.device == features.device and weight_saved.device == features.device,
             "features, grad_values and weight_saved must be on the same device")
    dev = features.device
    with torch.cuda.device(dev):
        out = torch.empty((h, w, vd), dtype=torch.float32, device=dev)
        lb, sb = _lib.workspace_sizes(h, w, pd, vd)
        if lattice is not None and lattice.matches(features, vd, same_object=not saved):
            state = 2 if lattice.used else 1
            buf, scratch, sbytes = lattice.buf, None, 0
        else:
            state = 0
            lattice = None
            buf = torch.empty(lb, dtype=torch.uint8, device=dev)
            scratch = torch.empty(sb, dtype=torch.uint8, device=dev)
            sbytes = sb
        rc = _lib.lib().plattice_backward(_ptr(out), _ptr(grad_values), _ptr(weight_saved),
                                          _ptr(features), _ptr(buf), lb, state, _ptr(scratch), sbytes,
                                          pd, vd, w, h, _stream(dev))
        if rc != _lib.OK:
            raise _lib.PlatticeError("plattice_backward", rc, f"h={h} w={w} pd={pd} vd={vd}")
        if lattice is not None:
            lattice.used = True
        if _CHECK and h * w > 0:
            chk = lattice if lattice is not None else Lattice(features, vd, buf, None)
            _sync_check(chk, "plattice_backward")
    return out


def _check_kept(lattice, t, name):
    _require(isinstance(lattice, Lattice), "lattice must be a Lattice from lattice_forward")
    _check_input(t, name)
    _require(t.dim() == 3, f"{name} must be [H, W, vd]")
    _require(t.dtype == torch.float32, f"{name} must be float32")
    _require((int(t.shape[0]), int(t.shape[1])) == (lattice.h, lattice.w),
             f"{name} must match the lattice's H, W")
    _require(t.device == lattice.device, f"{name} must be on the lattice's device")
    vd = int(t.shape[2])
    _check_dims(lattice.pd, vd)
    return vd


def lattice_filter(lattice, values):
    """Forward filter of ``values`` on a kept lattice (the lattice that
    :func:`lattice_forward` built, still holding its features' lattice; any
    vd): the same ``(weight [H,W,1], out [H,W,vd])`` as ``forward`` on those
    features, without rebuilding the lattice.  Calls on one lattice must run
    on one stream (they update its header)."""
    vd = _check_kept(lattice, values, "values")
    h, w, pd, dev = lattice.h, lattice.w, lattice.pd, lattice.device
    with torch.cuda.device(dev):
        out = torch.empty((h, w, vd), dtype=torch.float32, device=dev)
        weight = torch.empty((h, w, 1), dtype=torch.float32, device=dev)
        wsb = _lib.filter_workspace_size(h, w, pd, vd)
        ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
        rc = _lib.lib().plattice_filter(_ptr(weight), _ptr(out), _ptr(values), _ptr(lattice.buf),
                                        lattice.buf.numel(), _ptr(ws), wsb, pd, vd, w, h, _stream(dev))
        if rc != _lib.OK:
            raise _lib.PlatticeError("plattice_filter", rc, f"h={h} w={w} pd={pd} vd={vd}")
        if _CHECK and h * w > 0:
            _sync_check(lattice, "plattice_filter")
    return weight, out


def lattice_filter_backward(lattice, grad_values, weight_saved):
    """Value gradient of a :func:`lattice_filter` call on the same kept
    lattice, given that call's ``weight``; returns ``grad [H,W,vd]``."""
    vd = _check_kept(lattice, grad_values, "grad_values")
    _check_input(weight_saved, "weight_saved")
    _require(weight_saved.dim() == 3 and tuple(weight_saved.shape) == (lattice.h, lattice.w, 1),
             "weight_saved must be [H, W, 1]")
    _require(weight_saved.dtype == torch.float32, "weight_saved must be float32")
    h, w, pd, dev = lattice.h, lattice.w, lattice.pd, lattice.device
    with torch.cuda.device(dev):
        out = torch.empty((h, w, vd), dtype=torch.float32, device=dev)
        wsb = _lib.filter_workspace_size(h, w, pd, vd)
        ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
        rc = _lib.lib().plattice_filter_backward(_ptr(out), _ptr(grad_values), _ptr(weight_saved),
                                                 _ptr(lattice.buf), lattice.buf.numel(), _ptr(ws), wsb,
                                                 pd, vd, w, h, _stream(dev))
        if rc != _lib.OK:
            raise _lib.PlatticeError("plattice_filter_backward", rc, f"h={h} w={w} pd={pd} vd={vd}")
        if _CHECK and h * w > 0:
            _sync_check(lattice, "plattice_filter_backward")
    return out


def feature_grad(lattice, features, values, grad_out, weight, out):
    """Gradient ``[H,W,pd]`` of the forward filter with respect to ``features``
    for ``dL/dout = grad_out``, given the forward's ``weight`` and ``out`` on
    ``values`` and ``lattice``, the Lattice that forward built from ``features``
    (the reference returns no feature gradient).  The slope is that of the
    piecewise-linear filter inside each pixel's simplex."""
    _require(isinstance(lattice, Lattice), "lattice must be a Lattice from lattice_forward")
    _require(lattice.matches(features, lattice.vd, same_object=False),
             "lattice was not built from these features")
    for t, name in ((values, "values"), (grad_out, "grad_out"), (out, "out")):
        vd = _check_kept(lattice, t, name)
    _require(int(values.shape[2]) == int(grad_out.shape[2]) == int(out.shape[2]),
             "values, grad_out and out must have the same vd")
    _check_input(weight, "weight")
    _require(tuple(weight.shape) == (lattice.h, lattice.w, 1), "weight must be [H, W, 1]")
    h, w, pd, dev = lattice.h, lattice.w, lattice.pd, lattice.device
    with torch.cuda.device(dev):
        gf = torch.empty((h, w, pd), dtype=torch.float32, device=dev)
        wsb = _lib.feature_grad_workspace_size(h, w, pd, vd)
        ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
        rc = _lib.lib().plattice_feature_grad(_ptr(gf), _ptr(grad_out), _ptr(out), _ptr(weight), _ptr(values),
                                              _ptr(features), _ptr(lattice.buf), lattice.buf.numel(), _ptr(ws),
                                              wsb, pd, vd, w, h, _stream(dev))
        if rc != _lib.OK:
            raise _lib.PlatticeError("plattice_feature_grad", rc, f"h={h} w={w} pd={pd} vd={vd}")
        if _CHECK and h * w > 0:
            _sync_check(lattice, "plattice_feature_grad")
    return gf


class BatchLattice:
    """The lattices of a batch of images built by :func:`batch_forward`, kept
    for the batch's backward (one buffer, one lattice per image)."""

    __slots__ = ("buf", "shape", "vd", "device", "used", "_feat_ref", "_feat_version", "_feat_ptr",
                 "__weakref__")

    def __init__(self, features, vd, buf):
        self.buf = buf
        self.shape = tuple(int(s) for s in features.shape)
        self.vd = int(vd)
        self.device = features.device
        self.used = False
        self._feat_ref = weakref.ref(features)
        self._feat_version = features._version
        self._feat_ptr = features.data_ptr()

    def matches(self, features, vd, same_object=True):
        if same_object and self._feat_ref() is not features:
            return False
        return (features.data_ptr() == self._feat_ptr and int(vd) == self.vd
                and tuple(features.shape) == self.shape and features.device == self.device
                and (not same_object or features._version == self._feat_version))


def _check_batch(features, t, name):
    _check_input(features, "features")
    _check_input(t, name)
    _require(features.dim() == 4, "features must be [B, H, W, pd]")
    _require(t.dim() == 4, f"{name} must be [B, H, W, vd]")
    _require(features.dtype == torch.float32, "features must be float32")
    _require(t.dtype == torch.float32, f"{name} must be float32")
    _require(tuple(features.shape[:3]) == tuple(t.shape[:3]), f"features and {name} must have matching B, H, W")
    _require(t.device == features.device, f"features and {name} must be on the same device")
    b, h, w, pd = (int(x) for x in features.shape)
    vd = int(t.shape[3])
    _check_dims(pd, vd)
    return b, h, w, pd, vd


def batch_forward(features, values):
    """Forward filter of B images in one call, each image on its own lattice:
    ``features [B,H,W,pd]``, ``values [B,H,W,vd]`` -> ``(weight [B,H,W,1],
    out [B,H,W,vd], BatchLattice)``; the same per image as :func:`lattice_forward`."""
    b, h, w, pd, vd = _check_batch(features, values, "values")
    dev = features.device
    with torch.cuda.device(dev):
        out = torch.empty((b, h, w, vd), dtype=torch.float32, device=dev)
        weight = torch.empty((b, h, w, 1), dtype=torch.float32, device=dev)
        lb, sb = _lib.batch_workspace_sizes(b, h, w, pd, vd)
        buf = torch.empty(lb, dtype=torch.uint8, device=dev)
        scratch = torch.empty(sb, dtype=torch.uint8, device=dev)
        rc = _lib.lib().plattice_forward_batch(_ptr(weight), _ptr(out), _ptr(values), _ptr(features), _ptr(buf),
                                               lb, _ptr(scratch), sb, b, pd, vd, w, h, _stream(dev))
        if rc != _lib.OK:
            raise _lib.PlatticeError("plattice_forward_batch", rc, f"b={b} h={h} w={w} pd={pd} vd={vd}")
        lat = BatchLattice(features, vd, buf)
        if _CHECK and b * h * w > 0:
            _sync_check_batch(lat, b, h, w, pd, "plattice_forward_batch")
    return weight, out, lat


def batch_backward(features, grad_values, weight_saved, lattice=None, saved=False):
    """Value gradient of :func:`batch_forward`; reuses ``lattice`` when it was
    built from ``features`` as they are now, else rebuilds every image."""
    b, h, w, pd, vd = _check_batch(features, grad_values, "grad_values")
    _check_input(weight_saved, "weight_saved")
    _require(tuple(weight_saved.shape) == (b, h, w, 1), "weight_saved must be [B, H, W, 1]")
    _require(weight_saved.dtype == torch.float32, "weight_saved must be float32")
    dev = features.device
    with torch.cuda.device(dev):
        out = torch.empty((b, h, w, vd), dtype=torch.float32, device=dev)
        lb, sb = _lib.batch_workspace_sizes(b, h, w, pd, vd)
        if lattice is not None and lattice.matches(features, vd, same_object=not saved):
            state = 2 if lattice.used else 1
            buf, scratch, sbytes = lattice.buf, None, 0
        else:
            state = 0
            lattice = None
            buf = torch.empty(lb, dtype=torch.uint8, device=dev)
            scratch = torch.empty(sb, dtype=torch.uint8, device=dev)
            sbytes = sb
        rc = _lib.lib().plattice_backward_batch(_ptr(out), _ptr(grad_values), _ptr(weight_saved),
                                                _ptr(features), _ptr(buf), lb, state, _ptr(scratch), sbytes,
                                                b, pd, vd, w, h, _stream(dev))
        if rc != _lib.OK:
            raise _lib.PlatticeError("plattice_backward_batch", rc, f"b={b} h={h} w={w} pd={pd} vd={vd}")
        if lattice is not None:
            lattice.used = True
        if _CHECK and b * h * w > 0:
            _sync_check_batch(BatchLattice(features, vd, buf), b, h, w, pd, "plattice_backward_batch")
    return out


def _sync_check_batch(lat, b, h, w, pd, call):
    lb, _ = _lib.workspace_sizes(h, w, pd, lat.vd)
    stride = (lb + 255) & ~255
    for i in range(b):
        st = ctypes.c_int(0)
        rc = _lib.lib().plattice_lattice_info(ctypes.c_void_p(lat.buf.data_ptr() + i * stride),
                                              ctypes.byref(st), None, None, None, _stream(lat.device))
        if rc != _lib.OK:
            raise _lib.PlatticeError(call, rc, f"image {i}: device status bits {st.value:#x}")


# The most recent batch forward's lattices, for a standalone batch backward.
_last_batch = None


def forward_batch(features, values):
    """``forward`` over ``[B,H,W,...]`` -> ``[weight [B,H,W,1], out [B,H,W,vd]]``."""
    global _last_batch
    weight, out, lat = batch_forward(features, values)
    _last_batch = lat
    return [weight, out]


def backward_batch(features, grad_values, weight_saved):
    """``backward`` over ``[B,H,W,...]``; reuses the last batch forward's lattices."""
    return batch_backward(features, grad_values, weight_saved, _last_batch)


# The most recent forward's lattice, for a standalone backward on the same
# features (the reference's tests call forward then backward directly).
_last = None


def forward(features, values):
    """``PLOO.forward(features, values) -> [weight_out [H,W,1], out [H,W,vd]]``."""
    global _last
    weight, out, lat = lattice_forward(features, values)
    _last = lat
    return [weight, out]


def backward(features, grad_values, weight_saved):
    """``PLOO.backward(features, grad_values, weight_saved) -> grad [H,W,vd]``."""
    return lattice_backward(features, grad_values, weight_saved, _last)


def lattice_info(lattice):
    """Synchronise and read the lattice header: dict(status, m, u_total, cap_log2)."""
    st, m, u, cap = (ctypes.c_int(0) for _ in range(4))
    rc = _lib.lib().plattice_lattice_info(_ptr(lattice.buf), ctypes.byref(st), ctypes.byref(m),
                                          ctypes.byref(u), ctypes.byref(cap), _stream(lattice.device))
    if rc not in (_lib.OK, _lib.ERR_DEVICE):
        raise _lib.PlatticeError("plattice_lattice_info", rc)
    return {"status": st.value, "m": m.value, "u_total": u.value, "cap_log2": cap.value}


def vertex_keys(lattice):
    """Vertex keys [m, pd] int16 (device tensor) of a lattice built with
    ``lattice_forward(..., keep_scratch=True)``."""
    _require(lattice.scratch is not None, "vertex_keys needs a lattice built with keep_scratch=True")
    info = lattice_info(lattice)
    m = info["m"]
    keys = torch.empty((max(m, 1), lattice.pd), dtype=torch.int16, device=lattice.device)
    mm = ctypes.c_int(0)
    with torch.cuda.device(lattice.device):
        rc = _lib.lib().plattice_vertex_keys(_ptr(lattice.buf), _ptr(lattice.scratch), lattice.pd,
                                             lattice.vd, lattice.w, lattice.h, _ptr(keys), m,
                                             ctypes.byref(mm), _stream(lattice.device))
    if rc != _lib.OK:
        raise _lib.PlatticeError("plattice_vertex_keys", rc)
    return keys[:mm.value]


def set_lattice_precision(precision):
    """Lattice value precision of the blur passes of large lattices (more
    vertices than the blur grid keeps in registers): ``"fp32"`` (default) or
    ``"bf16"`` (rows stored as bfloat16 between passes, float arithmetic).
    Process-wide; applies to calls enqueued afterwards.  No counterpart in the
    reference, which computes in float only (permutohedral.cu:321-348)."""
    bits = {"fp32": 32, "bf16": 16}.get(precision)
    _require(bits is not None, f"lattice precision must be 'fp32' or 'bf16', got {precision!r}")
    rc = _lib.lib().plattice_set_lattice_precision(bits)
    if rc != _lib.OK:
        raise _lib.PlatticeError("plattice_set_lattice_precision", rc)


def get_lattice_precision():
    """``"fp32"`` or ``"bf16"``: the setting of set_lattice_precision."""
    return "bf16" if _lib.lib().plattice_get_lattice_precision() == 16 else "fp32"
