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

Device-side failures (a hash table too small, a bounded wait that gave up)
raise :class:`PlatticeError` at the first call after the failed call's kernels
have finished (or at :func:`check_device_status`).  Set the environment
variable PLATTICE_CHECK=1 to synchronise after every call and raise at once.

The hot paths (``lattice_forward``, ``lattice_backward``) do their checks with
one combined test first and build the reference's messages only on failure,
cache the workspace sizes per shape, and call the library directly on the
current device, so that their host cost stays a few microseconds above the
library call itself.
"""
import ctypes
import os
import weakref

import torch

from . import _lib

__all__ = ["forward", "backward", "Lattice", "lattice_forward", "lattice_backward",
           "lattice_filter", "lattice_filter_backward", "feature_grad", "BatchLattice", "batch_forward",
           "batch_backward", "forward_batch", "backward_batch", "lattice_info", "vertex_keys",
           "check_device_status", "prepare", "set_graph_cache", "graph_cache_stats", "set_keep_lattice",
           "get_keep_lattice"]

_CHECK = os.environ.get("PLATTICE_CHECK", "0") not in ("", "0")

# Whether the autograd Functions (PermutoLatticeFunction and its batch form)
# and forward / forward_batch keep the forward's lattice for the backward (the
# default: the backward skips the rebuild) or keep nothing and rebuild it in
# the backward, as the reference does (plattice.py:11-19,
# permutohedral.cu:615-635).  Off, a forward retains no device memory beyond
# its outputs, and the backward allocates the full lattice and scratch for its
# duration.  PLATTICE_KEEP_LATTICE=0 or set_keep_lattice(False).
_KEEP = os.environ.get("PLATTICE_KEEP_LATTICE", "1") not in ("", "0")

_F32 = torch.float32
_cur_dev = torch._C._cuda_getDevice
_raw_stream = torch._C._cuda_getCurrentRawStream
_L = None


def _lib_h():
    global _L
    if _L is None:
        _L = _lib.lib()
    return _L


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
    return t.data_ptr() if t is not None else None


def _stream(device):
    return _raw_stream(device.index)


_SIZES = {}


def _sizes(b, h, w, pd, vd):
    """(lattice bytes, full scratch bytes, kept-lattice scratch bytes), cached per shape."""
    key = (b, h, w, pd, vd)
    s = _SIZES.get(key)
    if s is None:
        lb, sb = _lib.batch_workspace_sizes(b, h, w, pd, vd)
        s = _SIZES[key] = (lb, sb, _lib.reuse_scratch_size(b, h, w, pd, vd))
    return s


_FILTER_WS = {}


def _filter_ws(h, w, pd, vd):
    key = (h, w, pd, vd)
    b = _FILTER_WS.get(key)
    if b is None:
        b = _FILTER_WS[key] = _lib.filter_workspace_size(h, w, pd, vd)
    return b


def _call(dev_index, fn, *args):
    """Library call with `dev_index` the current device (kernels launch on its stream)."""
    if _cur_dev() == dev_index:
        return fn(*args)
    with torch.cuda.device(dev_index):
        return fn(*args)


def _raise(call, rc, detail):
    raise _lib.PlatticeError(call, rc, detail)


class Lattice:
    """A lattice built on the device for one ``features`` tensor.

    Holds the lattice buffer (kept for backward calls) and optionally the
    scratch buffer of the build (needed by :func:`vertex_keys`).  A call on it
    that returns an error marks it ``broken`` (the call may have stopped part
    way, with the lattice's header in between two states): a backward then
    rebuilds, and the calls that need a kept lattice refuse it."""

    __slots__ = ("buf", "scratch", "h", "w", "pd", "vd", "device", "used", "broken", "_feat_ref",
                 "_feat_version", "_feat_ptr", "__weakref__")

    def __init__(self, features, vd, buf, scratch, shape=None):
        self.buf = buf
        self.scratch = scratch
        self.h, self.w, self.pd = shape if shape is not None else (int(s) for s in features.shape)
        self.vd = int(vd)
        self.device = features.device
        self.used = False
        self.broken = False
        self._feat_ref = weakref.ref(features)
        self._feat_version = features._version
        self._feat_ptr = features.data_ptr()

    def matches(self, features, vd, same_object=True):
        """True when this lattice was built from ``features`` as it is now
        (and no call on it has failed since).  ``same_object=False`` drops the
        identity test, for callers (autograd's saved tensors) that hand back a
        new tensor object over the same, version-checked storage.  A lattice
        serves every vd."""
        if self.broken or (same_object and self._feat_ref() is not features):
            return False
        return (features.data_ptr() == self._feat_ptr
                and tuple(features.shape) == (self.h, self.w, self.pd)
                and features.device == self.device
                and (not same_object or features._version == self._feat_version))


def _sync_check(lat, call):
    st = ctypes.c_int(0)
    rc = _lib_h().plattice_lattice_info(_ptr(lat.buf), ctypes.byref(st), None, None, None,
                                        _stream(lat.device))
    if rc != _lib.OK:
        _raise(call, rc, f"device status bits {st.value:#x}")


def _forward_checks(features, values):
    _check_input(features, "features")
    _check_input(values, "values")
    _require(features.dim() == 3, "features must be [H, W, pd]")
    _require(values.dim() == 3, "values must be [H, W, vd]")
    _require(features.dtype == torch.float32, "features must be float32")
    _require(values.dtype == torch.float32, "values must be float32")
    _require(features.shape[0] == values.shape[0] and features.shape[1] == values.shape[1],
             "features and values must have matching H, W")
    _check_dims(int(features.shape[2]), int(values.shape[2]))
    _require(values.device == features.device, "features and values must be on the same device")


def lattice_forward(features, values, keep_scratch=False):
    """Forward filter; returns ``(weight [H,W,1], out [H,W,vd], Lattice)``."""
    if not (isinstance(features, torch.Tensor) and isinstance(values, torch.Tensor)
            and features.is_cuda and values.is_cuda and len(fs := features.shape) == 3
            and len(vs := values.shape) == 3
            and features.dtype is _F32 and values.dtype is _F32
            and fs[0] == vs[0] and fs[1] == vs[1] and 1 <= fs[2] <= 16 and 1 <= vs[2] <= 8
            and features.is_contiguous() and values.is_contiguous()
            and values.device == features.device):
        _forward_checks(features, values)
    h, w, pd = features.shape
    vd = values.shape[2]
    dev = features.device
    out = torch.empty((h, w, vd), dtype=_F32, device=dev)
    weight = torch.empty((h, w, 1), dtype=_F32, device=dev)
    lb, sb, _ = _sizes(1, h, w, pd, vd)
    buf = torch.empty(lb, dtype=torch.uint8, device=dev)
    scratch = torch.empty(sb, dtype=torch.uint8, device=dev)
    rc = _call(dev.index, _lib_h().plattice_forward, weight.data_ptr(), out.data_ptr(), values.data_ptr(),
               features.data_ptr(), buf.data_ptr(), lb, scratch.data_ptr(), sb, pd, vd, w, h,
               _raw_stream(dev.index))
    if rc:
        _raise("plattice_forward", rc, f"h={h} w={w} pd={pd} vd={vd}")
    lat = Lattice(features, vd, buf, scratch if keep_scratch else None, (h, w, pd))
    if _CHECK and h * w > 0:
        _sync_check(lat, "plattice_forward")
    return weight, out, lat


def _backward_checks(features, grad_values, weight_saved):
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
    _check_dims(int(features.shape[2]), int(grad_values.shape[2]))
    _require(grad_values.device == features.device and weight_saved.device == features.device,
             "features, grad_values and weight_saved must be on the same device")


def lattice_backward(features, grad_values, weight_saved, lattice=None, saved=False):
    """Value gradient; reuses ``lattice`` when it was built from ``features``
    as they are now, else rebuilds.  ``saved=True`` when ``features`` comes
    from autograd's saved tensors (whose version check already guarantees
    they are unmodified).  Returns ``grad [H,W,vd]``."""
    if not (isinstance(features, torch.Tensor) and isinstance(grad_values, torch.Tensor)
            and isinstance(weight_saved, torch.Tensor)
            and features.is_cuda and grad_values.is_cuda and weight_saved.is_cuda
            and len(fs := features.shape) == 3 and len(gs := grad_values.shape) == 3
            and len(ws := weight_saved.shape) == 3 and ws[2] == 1
            and features.dtype is _F32 and grad_values.dtype is _F32 and weight_saved.dtype is _F32
            and fs[0] == gs[0] == ws[0] and fs[1] == gs[1] == ws[1]
            and 1 <= fs[2] <= 16 and 1 <= gs[2] <= 8
            and features.is_contiguous() and grad_values.is_contiguous() and weight_saved.is_contiguous()
            and grad_values.device == features.device and weight_saved.device == features.device):
        _backward_checks(features, grad_values, weight_saved)
    h, w, pd = features.shape
    vd = grad_values.shape[2]
    dev = features.device
    out = torch.empty((h, w, vd), dtype=_F32, device=dev)
    lb, sb, rb = _sizes(1, h, w, pd, vd)
    if lattice is not None and lattice.matches(features, vd, same_object=not saved):
        state = 2 if lattice.used else 1
        buf, sbytes = lattice.buf, rb
    else:
        state = 0
        lattice = None
        buf = torch.empty(lb, dtype=torch.uint8, device=dev)
        sbytes = sb
    scratch = torch.empty(sbytes, dtype=torch.uint8, device=dev)
    rc = _call(dev.index, _lib_h().plattice_backward, out.data_ptr(), grad_values.data_ptr(),
               weight_saved.data_ptr(), features.data_ptr(), buf.data_ptr(), lb, state, scratch.data_ptr(),
               sbytes, pd, vd, w, h, _raw_stream(dev.index))
    if rc:
        if lattice is not None:
            lattice.broken = True
        _raise("plattice_backward", rc, f"h={h} w={w} pd={pd} vd={vd}")
    if lattice is not None:
        lattice.used = True
    if _CHECK and h * w > 0:
        chk = lattice if lattice is not None else Lattice(features, vd, buf, None)
        _sync_check(chk, "plattice_backward")
    return out


def _check_kept(lattice, t, name):
    _require(isinstance(lattice, Lattice), "lattice must be a Lattice from lattice_forward")
    _require(not lattice.broken, "lattice is unusable after a failed call on it: build it again")
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
    out = torch.empty((h, w, vd), dtype=_F32, device=dev)
    weight = torch.empty((h, w, 1), dtype=_F32, device=dev)
    wsb = _filter_ws(h, w, pd, vd)
    ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
    rc = _call(dev.index, _lib_h().plattice_filter, weight.data_ptr(), out.data_ptr(), values.data_ptr(),
               lattice.buf.data_ptr(), lattice.buf.numel(), ws.data_ptr(), wsb, pd, vd, w, h,
               _raw_stream(dev.index))
    if rc:
        lattice.broken = True
        _raise("plattice_filter", rc, f"h={h} w={w} pd={pd} vd={vd}")
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
    out = torch.empty((h, w, vd), dtype=_F32, device=dev)
    wsb = _filter_ws(h, w, pd, vd)
    ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
    rc = _call(dev.index, _lib_h().plattice_filter_backward, out.data_ptr(), grad_values.data_ptr(),
               weight_saved.data_ptr(), lattice.buf.data_ptr(), lattice.buf.numel(), ws.data_ptr(), wsb,
               pd, vd, w, h, _raw_stream(dev.index))
    if rc:
        lattice.broken = True
        _raise("plattice_filter_backward", rc, f"h={h} w={w} pd={pd} vd={vd}")
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
    _require(not lattice.broken, "lattice is unusable after a failed call on it: build it again")
    _require(lattice.matches(features, lattice.vd, same_object=False),
             "lattice was not built from these features")
    for t, name in ((values, "values"), (grad_out, "grad_out"), (out, "out")):
        vd = _check_kept(lattice, t, name)
    _require(int(values.shape[2]) == int(grad_out.shape[2]) == int(out.shape[2]),
             "values, grad_out and out must have the same vd")
    _check_input(weight, "weight")
    _require(tuple(weight.shape) == (lattice.h, lattice.w, 1), "weight must be [H, W, 1]")
    h, w, pd, dev = lattice.h, lattice.w, lattice.pd, lattice.device
    gf = torch.empty((h, w, pd), dtype=_F32, device=dev)
    wsb = _lib.feature_grad_workspace_size(h, w, pd, vd)
    ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
    rc = _call(dev.index, _lib_h().plattice_feature_grad, gf.data_ptr(), grad_out.data_ptr(), out.data_ptr(),
               weight.data_ptr(), values.data_ptr(), features.data_ptr(), lattice.buf.data_ptr(),
               lattice.buf.numel(), ws.data_ptr(), wsb, pd, vd, w, h, _raw_stream(dev.index))
    if rc:
        lattice.broken = True
        _raise("plattice_feature_grad", rc, f"h={h} w={w} pd={pd} vd={vd}")
    if _CHECK and h * w > 0:
        _sync_check(lattice, "plattice_feature_grad")
    return gf


class BatchLattice:
    """The lattice of a batch of images built by :func:`batch_forward`, kept
    for the batch's backward (one buffer; the images' vertices are kept apart
    by the image index in the key hash)."""

    __slots__ = ("buf", "shape", "vd", "device", "used", "broken", "_feat_ref", "_feat_version", "_feat_ptr",
                 "__weakref__")

    def __init__(self, features, vd, buf):
        self.buf = buf
        self.shape = tuple(int(s) for s in features.shape)
        self.vd = int(vd)
        self.device = features.device
        self.used = False
        self.broken = False   # a call on it returned an error: the backward rebuilds
        self._feat_ref = weakref.ref(features)
        self._feat_version = features._version
        self._feat_ptr = features.data_ptr()

    def matches(self, features, vd, same_object=True):
        if self.broken or (same_object and self._feat_ref() is not features):
            return False
        return (features.data_ptr() == self._feat_ptr
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
    out = torch.empty((b, h, w, vd), dtype=_F32, device=dev)
    weight = torch.empty((b, h, w, 1), dtype=_F32, device=dev)
    lb, sb, _ = _sizes(b, h, w, pd, vd)
    buf = torch.empty(lb, dtype=torch.uint8, device=dev)
    scratch = torch.empty(sb, dtype=torch.uint8, device=dev)
    rc = _call(dev.index, _lib_h().plattice_forward_batch, weight.data_ptr(), out.data_ptr(), values.data_ptr(),
               features.data_ptr(), buf.data_ptr(), lb, scratch.data_ptr(), sb, b, pd, vd, w, h,
               _raw_stream(dev.index))
    if rc:
        _raise("plattice_forward_batch", rc, f"b={b} h={h} w={w} pd={pd} vd={vd}")
    lat = BatchLattice(features, vd, buf)
    if _CHECK and b * h * w > 0:
        _sync_check(lat, "plattice_forward_batch")
    return weight, out, lat


def batch_backward(features, grad_values, weight_saved, lattice=None, saved=False):
    """Value gradient of :func:`batch_forward`; reuses ``lattice`` when it was
    built from ``features`` as they are now, else rebuilds every image."""
    b, h, w, pd, vd = _check_batch(features, grad_values, "grad_values")
    _check_input(weight_saved, "weight_saved")
    _require(tuple(weight_saved.shape) == (b, h, w, 1), "weight_saved must be [B, H, W, 1]")
    _require(weight_saved.dtype == torch.float32, "weight_saved must be float32")
    dev = features.device
    out = torch.empty((b, h, w, vd), dtype=_F32, device=dev)
    lb, sb, rb = _sizes(b, h, w, pd, vd)
    if lattice is not None and lattice.matches(features, vd, same_object=not saved):
        state = 2 if lattice.used else 1
        buf, sbytes = lattice.buf, rb
    else:
        state = 0
        lattice = None
        buf = torch.empty(lb, dtype=torch.uint8, device=dev)
        sbytes = sb
    scratch = torch.empty(sbytes, dtype=torch.uint8, device=dev)
    rc = _call(dev.index, _lib_h().plattice_backward_batch, out.data_ptr(), grad_values.data_ptr(),
               weight_saved.data_ptr(), features.data_ptr(), buf.data_ptr(), lb, state, scratch.data_ptr(),
               sbytes, b, pd, vd, w, h, _raw_stream(dev.index))
    if rc:
        if lattice is not None:
            lattice.broken = True
        _raise("plattice_backward_batch", rc, f"b={b} h={h} w={w} pd={pd} vd={vd}")
    if lattice is not None:
        lattice.used = True
    if _CHECK and b * h * w > 0:
        _sync_check(BatchLattice(features, vd, buf), "plattice_backward_batch")
    return out


# The most recent batch forward's lattice, for a standalone batch backward.
_last_batch = None


def forward_batch(features, values):
    """``forward`` over ``[B,H,W,...]`` -> ``[weight [B,H,W,1], out [B,H,W,vd]]``."""
    global _last_batch
    weight, out, lat = batch_forward(features, values)
    _last_batch = lat if _KEEP else None
    return [weight, out]


def backward_batch(features, grad_values, weight_saved):
    """``backward`` over ``[B,H,W,...]``; reuses the last batch forward's lattice."""
    return batch_backward(features, grad_values, weight_saved, _last_batch)


# The most recent forward's lattice, for a standalone backward on the same
# features (the reference's tests call forward then backward directly).
_last = None


def forward(features, values):
    """``PLOO.forward(features, values) -> [weight_out [H,W,1], out [H,W,vd]]``."""
    global _last
    weight, out, lat = lattice_forward(features, values)
    _last = lat if _KEEP else None
    return [weight, out]


def backward(features, grad_values, weight_saved):
    """``PLOO.backward(features, grad_values, weight_saved) -> grad [H,W,vd]``."""
    return lattice_backward(features, grad_values, weight_saved, _last)


def check_device_status():
    """Raise :class:`PlatticeError` if an earlier call's kernels finished with
    a device-side failure not yet reported (does not synchronise)."""
    rc = _lib_h().plattice_poll_status()
    if rc:
        _raise("plattice_poll_status", rc, "")


def prepare(pd, vd, device=None):
    """Do once, on ``device``'s context, what a first call for (pd, vd) would
    do besides filtering: kernel attributes, occupancy queries, kernel loading."""
    _check_dims(pd, vd)
    idx = torch.cuda.current_device() if device is None else torch.device(device).index
    rc = _call(idx, _lib_h().plattice_prepare, pd, vd)
    if rc:
        _raise("plattice_prepare", rc, f"pd={pd} vd={vd}")


def lattice_info(lattice):
    """Synchronise and read the lattice header: dict(status, m, u_total, cap_log2)."""
    st, m, u, cap = (ctypes.c_int(0) for _ in range(4))
    rc = _lib_h().plattice_lattice_info(_ptr(lattice.buf), ctypes.byref(st), ctypes.byref(m),
                                        ctypes.byref(u), ctypes.byref(cap), _stream(lattice.device))
    if rc not in (_lib.OK, _lib.ERR_DEVICE):
        _raise("plattice_lattice_info", rc, "")
    return {"status": st.value, "m": m.value, "u_total": u.value, "cap_log2": cap.value}


def vertex_keys(lattice):
    """Vertex keys [m, pd] int16 (device tensor) of a lattice built with
    ``lattice_forward(..., keep_scratch=True)``."""
    _require(lattice.scratch is not None, "vertex_keys needs a lattice built with keep_scratch=True")
    info = lattice_info(lattice)
    m = info["m"]
    keys = torch.empty((max(m, 1), lattice.pd), dtype=torch.int16, device=lattice.device)
    mm = ctypes.c_int(0)
    rc = _call(lattice.device.index, _lib_h().plattice_vertex_keys, _ptr(lattice.buf), _ptr(lattice.scratch),
               lattice.pd, lattice.vd, lattice.w, lattice.h, _ptr(keys), m, ctypes.byref(mm),
               _stream(lattice.device))
    if rc != _lib.OK:
        _raise("plattice_vertex_keys", rc, "")
    return keys[:mm.value]


def set_lattice_precision(precision):
    """Lattice value precision of the blur passes of large lattices (more
    vertices than the blur grid keeps in registers): ``"fp32"`` (default) or
    ``"bf16"`` (rows stored as bfloat16 between passes, float arithmetic).
    Process-wide; applies to calls enqueued afterwards.  No counterpart in the
    reference, which computes in float only (permutohedral.cu:321-348)."""
    bits = {"fp32": 32, "bf16": 16}.get(precision)
    _require(bits is not None, f"lattice precision must be 'fp32' or 'bf16', got {precision!r}")
    rc = _lib_h().plattice_set_lattice_precision(bits)
    if rc != _lib.OK:
        _raise("plattice_set_lattice_precision", rc, "")


def set_keep_lattice(keep):
    """Keep the forward's lattice for the backward (``True``, the default) or,
    as the reference does, keep nothing and rebuild it in the backward
    (``False``): no device memory retained between the two (482 MiB at
    1024 x 1024 pd 5 otherwise), for a rebuild in every backward.  Applies to
    the forwards made after it: PermutoLatticeFunction,
    PermutoLatticeBatchFunction, forward and forward_batch.  Results do not
    depend on it (within the float tolerance of the splat's summation order)."""
    global _KEEP
    _require(isinstance(keep, bool), "keep must be a bool")
    _KEEP = keep


def get_keep_lattice():
    """The setting of :func:`set_keep_lattice`."""
    return _KEEP


def get_lattice_precision():
    """``"fp32"`` or ``"bf16"``: the setting of set_lattice_precision."""
    return "bf16" if _lib_h().plattice_get_lattice_precision() == 16 else "fp32"


def set_graph_cache(entries):
    """Graphs kept per CUDA context for calls repeated with the same buffers
    (``plattice_set_graph_cache``): such a call is captured into a CUDA graph
    the second time and replayed afterwards, one launch on the host instead of
    one per kernel.  0 turns it off; the default is 16 (0 when the
    environment variable PLATTICE_GRAPHS is "0").  Results do not depend on it."""
    _require(isinstance(entries, int) and entries >= 0, "entries must be a non-negative int")
    rc = _lib_h().plattice_set_graph_cache(entries)
    if rc != _lib.OK:
        _raise("plattice_set_graph_cache", rc, "")


def graph_cache_stats():
    """``(captures, replays)`` of call graphs so far, process-wide."""
    c, r = ctypes.c_longlong(0), ctypes.c_longlong(0)
    _lib_h().plattice_graph_cache_stats(ctypes.byref(c), ctypes.byref(r))
    return c.value, r.value
