"""ctypes binding of libplattice_b200.so (the C ABI of include/plattice.h).

The library is built in-tree by ``python -m plattice_pytorch_b200.build`` (or
``__graft_entry__.build()``).  There is no fallback: when the library is
missing or cannot be loaded, every call raises.
"""
import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libplattice_b200.so")

OK, ERR_INVALID, ERR_WORKSPACE, ERR_CUDA, ERR_DEVICE = 0, 1, 2, 3, 4
DEV_TABLE_FULL, DEV_WAIT_LIMIT, DEV_ROUND_LIMIT = 2, 4, 8
ABI_VERSION = 5

_lock = threading.Lock()
_lib = None


class PlatticeError(RuntimeError):
    """A failure reported by the CUDA library."""

    def __init__(self, call, status, detail=""):
        self.status = status
        msg = f"{call} failed: {error_string(status)} (status {status})"
        if detail:
            msg += f"; {detail}"
        if status in (ERR_CUDA, ERR_DEVICE):
            try:
                msg += f"; {lib().plattice_last_error_detail().decode()}"
            except ImportError:
                pass
        super().__init__(msg)


def lib():
    """Load (once) and return the ctypes library handle."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build the CUDA library with "
                "`python -m plattice_pytorch_b200.build` (nvcc, sm_100a)")
        L = ctypes.CDLL(LIB_PATH)
        P, I, S = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
        L.plattice_abi_version.restype = I
        L.plattice_abi_version.argtypes = []
        L.plattice_error_string.restype = ctypes.c_char_p
        L.plattice_error_string.argtypes = [I]
        L.plattice_last_error_detail.restype = ctypes.c_char_p
        L.plattice_last_error_detail.argtypes = []
        L.plattice_workspace_sizes.restype = I
        L.plattice_workspace_sizes.argtypes = [I, I, I, I, ctypes.POINTER(S), ctypes.POINTER(S)]
        L.plattice_forward.restype = I
        L.plattice_forward.argtypes = [P, P, P, P, P, S, P, S, I, I, I, I, P]
        L.plattice_backward.restype = I
        L.plattice_backward.argtypes = [P, P, P, P, P, S, I, P, S, I, I, I, I, P]
        L.plattice_batch_workspace_sizes.restype = I
        L.plattice_batch_workspace_sizes.argtypes = [I, I, I, I, I, ctypes.POINTER(S), ctypes.POINTER(S)]
        L.plattice_forward_batch.restype = I
        L.plattice_forward_batch.argtypes = [P, P, P, P, P, S, P, S, I, I, I, I, I, P]
        L.plattice_backward_batch.restype = I
        L.plattice_backward_batch.argtypes = [P, P, P, P, P, S, I, P, S, I, I, I, I, I, P]
        L.plattice_feature_grad_workspace_size.restype = I
        L.plattice_feature_grad_workspace_size.argtypes = [I, I, I, I, ctypes.POINTER(S)]
        L.plattice_feature_grad.restype = I
        L.plattice_feature_grad.argtypes = [P, P, P, P, P, P, P, S, P, S, I, I, I, I, P]
        L.plattice_reuse_scratch_size.restype = I
        L.plattice_reuse_scratch_size.argtypes = [I, I, I, I, I, ctypes.POINTER(S)]
        L.plattice_poll_status.restype = I
        L.plattice_poll_status.argtypes = []
        L.plattice_prepare.restype = I
        L.plattice_prepare.argtypes = [I, I]
        L.plattice_set_graph_cache.restype = I
        L.plattice_set_graph_cache.argtypes = [I]
        L.plattice_graph_cache_stats.restype = None
        L.plattice_graph_cache_stats.argtypes = [ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong)]
        L.plattice_forward_noalloc.restype = I
        L.plattice_forward_noalloc.argtypes = [P, P, P, P, I, I, I, I, P]
        L.plattice_noalloc_capacity.restype = S
        L.plattice_noalloc_capacity.argtypes = []
        L.plattice_noalloc_error_detail.restype = ctypes.c_char_p
        L.plattice_noalloc_error_detail.argtypes = []
        L.plattice_noalloc_status.restype = I
        L.plattice_noalloc_status.argtypes = [ctypes.POINTER(I), ctypes.POINTER(I), P]
        L.plattice_filter_workspace_size.restype = I
        L.plattice_filter_workspace_size.argtypes = [I, I, I, I, ctypes.POINTER(S)]
        L.plattice_filter.restype = I
        L.plattice_filter.argtypes = [P, P, P, P, S, P, S, I, I, I, I, P]
        L.plattice_filter_backward.restype = I
        L.plattice_filter_backward.argtypes = [P, P, P, P, S, P, S, I, I, I, I, P]
        L.plattice_lattice_info.restype = I
        L.plattice_lattice_info.argtypes = [P, ctypes.POINTER(I), ctypes.POINTER(I),
                                            ctypes.POINTER(I), ctypes.POINTER(I), P]
        L.plattice_vertex_keys.restype = I
        L.plattice_vertex_keys.argtypes = [P, P, I, I, I, I, P, I, ctypes.POINTER(I), P]
        L.plattice_debug_set_table_cap_log2.restype = None
        L.plattice_debug_set_table_cap_log2.argtypes = [I]
        L.plattice_debug_set_miss_filter_log2.restype = None
        L.plattice_debug_set_miss_filter_log2.argtypes = [I]
        L.plattice_set_lattice_precision.restype = I
        L.plattice_set_lattice_precision.argtypes = [I]
        L.plattice_get_lattice_precision.restype = I
        L.plattice_get_lattice_precision.argtypes = []
        L.plattice_debug_set_blur_streaming.restype = None
        L.plattice_debug_set_blur_streaming.argtypes = [I]
        L.plattice_profile_enable.restype = None
        L.plattice_profile_enable.argtypes = [I]
        L.plattice_profile_read.restype = I
        L.plattice_profile_read.argtypes = [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(I), I]
        L.plattice_profile_stage_name.restype = ctypes.c_char_p
        L.plattice_profile_stage_name.argtypes = [I]
        v = L.plattice_abi_version()
        if v != ABI_VERSION:
            raise ImportError(f"{LIB_PATH} has ABI version {v}, expected {ABI_VERSION}: rebuild it")
        _lib = L
    return _lib


def error_string(status):
    try:
        return lib().plattice_error_string(int(status)).decode()
    except ImportError:
        return "unknown"


def workspace_sizes(h, w, pd, vd):
    lb, sb = ctypes.c_size_t(0), ctypes.c_size_t(0)
    rc = lib().plattice_workspace_sizes(h, w, pd, vd, ctypes.byref(lb), ctypes.byref(sb))
    if rc != OK:
        raise PlatticeError("plattice_workspace_sizes", rc, f"h={h} w={w} pd={pd} vd={vd}")
    return lb.value, sb.value


def batch_workspace_sizes(b, h, w, pd, vd):
    lb, sb = ctypes.c_size_t(0), ctypes.c_size_t(0)
    rc = lib().plattice_batch_workspace_sizes(b, h, w, pd, vd, ctypes.byref(lb), ctypes.byref(sb))
    if rc != OK:
        raise PlatticeError("plattice_batch_workspace_sizes", rc, f"b={b} h={h} w={w} pd={pd} vd={vd}")
    return lb.value, sb.value


def reuse_scratch_size(b, h, w, pd, vd):
    """Scratch bytes of a call on a kept lattice of b images (the front part
    of the full scratch: the value rows of its blur)."""
    n = ctypes.c_size_t(0)
    rc = lib().plattice_reuse_scratch_size(b, h, w, pd, vd, ctypes.byref(n))
    if rc != OK:
        raise PlatticeError("plattice_reuse_scratch_size", rc, f"b={b} h={h} w={w} pd={pd} vd={vd}")
    return n.value


def feature_grad_workspace_size(h, w, pd, vd):
    b = ctypes.c_size_t(0)
    rc = lib().plattice_feature_grad_workspace_size(h, w, pd, vd, ctypes.byref(b))
    if rc != OK:
        raise PlatticeError("plattice_feature_grad_workspace_size", rc, f"h={h} w={w} pd={pd} vd={vd}")
    return b.value


def filter_workspace_size(h, w, pd, vd):
    b = ctypes.c_size_t(0)
    rc = lib().plattice_filter_workspace_size(h, w, pd, vd, ctypes.byref(b))
    if rc != OK:
        raise PlatticeError("plattice_filter_workspace_size", rc, f"h={h} w={w} pd={pd} vd={vd}")
    return b.value


PROFILE_STAGES = 14


def profile_enable(on=True, groups=False):
    """Bracket every kernel launch with CUDA events, or with ``groups=True``
    only the launch groups (build, forward filter, backward filter); see
    profile_read."""
    lib().plattice_profile_enable((2 if groups else 1) if on else 0)


def profile_read():
    """Wait for the recorded launches; return {stage: (total_ms, launches)} and clear."""
    ms = (ctypes.c_double * PROFILE_STAGES)()
    n = (ctypes.c_int * PROFILE_STAGES)()
    rc = lib().plattice_profile_read(ms, n, PROFILE_STAGES)
    if rc != OK:
        raise PlatticeError("plattice_profile_read", rc)
    return {lib().plattice_profile_stage_name(i).decode(): (ms[i], n[i]) for i in range(PROFILE_STAGES)}
