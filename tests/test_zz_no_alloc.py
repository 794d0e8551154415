"""The forward entry point for callers that cannot allocate device memory.

plattice_forward_noalloc serves code that must not call cudaMalloc (or a
caching allocator) when it runs the filter -- a plugin whose host owns every
device allocation, a real-time loop that forbids allocation after start-up,
code that runs while a memory pool is frozen.  It keeps its lattice and
scratch in a fixed array inside the library, so the caller only hands over
inputs and outputs.  These tests call it through the C ABI several times in a
row on different images, two of the same shape among them (the array keeps
the previous call's contents, which must not leak into the next result), and
compare each result with the regular entry point, which takes its workspace
from PyTorch; they read the device status word back from the array after each
call, and check that an image too large for the array is refused with an
error instead of being run.

This file is collected last on purpose: a failure here leaves every other
test already run.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, allclose_report

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 5e-6


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from plattice_pytorch_b200 import _lib
    L = _lib.lib()
    P, I = ctypes.c_void_p, ctypes.c_int
    L.plattice_forward_noalloc.argtypes = [P, P, P, P, I, I, I, I, P]
    L.plattice_forward_noalloc.restype = I
    L.plattice_noalloc_capacity.argtypes = []
    L.plattice_noalloc_capacity.restype = ctypes.c_size_t
    L.plattice_noalloc_error_detail.argtypes = []
    L.plattice_noalloc_error_detail.restype = ctypes.c_char_p
    L.plattice_noalloc_status.argtypes = [ctypes.POINTER(I), ctypes.POINTER(I), P]
    L.plattice_noalloc_status.restype = I
    return L


def _noalloc_forward(L, f, v):
    h, w, pd = f.shape
    vd = v.shape[2]
    out = torch.empty((h, w, vd), dtype=torch.float32, device=f.device)
    wo = torch.empty((h, w, 1), dtype=torch.float32, device=f.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(f.device).cuda_stream)
    rc = L.plattice_forward_noalloc(ctypes.c_void_p(wo.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                    ctypes.c_void_p(v.data_ptr()), ctypes.c_void_p(f.data_ptr()),
                                    pd, vd, w, h, stream)
    assert rc == 0, (rc, L.plattice_noalloc_error_detail().decode())
    return wo, out


def _case(name, dev):
    d = np.load(os.path.join(GOLDEN, name))
    return (torch.from_numpy(d["features"]).to(dev), torch.from_numpy(d["values"]).to(dev))


def _noalloc_status(L, dev):
    st, m = ctypes.c_int(-1), ctypes.c_int(-1)
    rc = L.plattice_noalloc_status(ctypes.byref(st), ctypes.byref(m),
                                   ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    return rc, st.value, m.value


def test_calls_in_a_row_match_the_allocating_entry_point(lib):
    """A, B, A on one shape (the array keeps the previous call's hash table,
    counters and rows at the same offsets, so a part that is not cleared would
    show), then another shape and pd; each result equals the allocating entry
    point's, and the status read from the array is clean with the same vertex
    count."""
    from plattice_pytorch_b200 import PLOO
    from plattice_pytorch_b200.workloads import make_workload
    dev = torch.device("cuda:0")
    a = _case("ref_blobs64_pd5_vd3.npz", dev)
    w = make_workload("blobs64_pd5_vd3", seed=9)
    b = (torch.from_numpy(w["features"]).to(dev), torch.from_numpy(w["values"]).to(dev))
    c = _case("ref_randn24x20_pd16_vd1.npz", dev)
    for f, v in (a, b, a, c):
        wo_n, out_n = _noalloc_forward(lib, f, v)
        rc, st, m = _noalloc_status(lib, dev)
        wo_r, out_r, lat = PLOO.lattice_forward(f, v)
        torch.cuda.synchronize()
        assert rc == 0 and st == 0
        assert m == PLOO.lattice_info(lat)["m"]
        assert allclose_report(out_n.cpu().numpy(), out_r.cpu().numpy(), RTOL, ATOL) <= 1.0
        assert allclose_report(wo_n.cpu().numpy(), wo_r.cpu().numpy(), RTOL, ATOL) <= 1.0


def test_workspace_larger_than_the_array_is_refused(lib):
    from plattice_pytorch_b200 import _lib
    dev = torch.device("cuda:0")
    h = w = 1024
    f = torch.zeros((h, w, 5), dtype=torch.float32, device=dev)
    v = torch.zeros((h, w, 3), dtype=torch.float32, device=dev)
    out = torch.empty((h, w, 3), dtype=torch.float32, device=dev)
    wo = torch.empty((h, w, 1), dtype=torch.float32, device=dev)
    lb, sb = _lib.workspace_sizes(h, w, 5, 3)
    assert lb + sb > lib.plattice_noalloc_capacity()
    rc = lib.plattice_forward_noalloc(ctypes.c_void_p(wo.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                      ctypes.c_void_p(v.data_ptr()), ctypes.c_void_p(f.data_ptr()),
                                      5, 3, w, h, ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    assert rc == _lib.ERR_WORKSPACE
    assert b"fixed array" in lib.plattice_noalloc_error_detail()
    # the next call's message does not repeat it
    f, v = _case("ref_blobs64_pd5_vd3.npz", dev)
    _noalloc_forward(lib, f, v)
    assert lib.plattice_noalloc_error_detail() == b""
