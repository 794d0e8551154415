"""Call graphs: a forward or backward repeated with the same buffers runs as
a captured CUDA graph from its second occurrence on (plattice_set_graph_cache).

The checker is the reference-generated golden case (and the direct launches
with graphs turned off): every call of a sequence on fixed buffers -- the
first run directly, the second captured and launched, the later ones
replayed -- gives the
golden output, normaliser and value gradient within 1e-5 relative + 5e-6
absolute; replays are counted; a device failure of a replayed call is still
reported on the next call, since the replay points the status-reporting
kernel at the call's own status slot.
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
    return _lib.lib()


class Buffers:
    """Fixed device buffers of one golden case, for calls through the C ABI."""

    def __init__(self, name, dev):
        from plattice_pytorch_b200 import _lib
        d = np.load(os.path.join(GOLDEN, name))
        self.d = d
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        self.f, self.v, self.g = t(d["features"]), t(d["values"]), t(d["grad"])
        self.h, self.w, self.pd = self.f.shape
        self.vd = self.v.shape[2]
        self.lb, self.sb = _lib.workspace_sizes(self.h, self.w, self.pd, self.vd)
        self.lat = torch.empty(self.lb, dtype=torch.uint8, device=dev)
        self.scr = torch.empty(self.sb, dtype=torch.uint8, device=dev)
        self.out = torch.empty((self.h, self.w, self.vd), device=dev)
        self.wo = torch.empty((self.h, self.w, 1), device=dev)
        self.gout = torch.empty((self.h, self.w, self.vd), device=dev)
        self.stream = torch.cuda.current_stream(dev).cuda_stream

    def forward(self, L):
        return L.plattice_forward(self.wo.data_ptr(), self.out.data_ptr(), self.v.data_ptr(), self.f.data_ptr(),
                                  self.lat.data_ptr(), self.lb, self.scr.data_ptr(), self.sb, self.pd, self.vd,
                                  self.w, self.h, self.stream)

    def backward(self, L, state):
        return L.plattice_backward(self.gout.data_ptr(), self.g.data_ptr(), self.wo.data_ptr(), self.f.data_ptr(),
                                   self.lat.data_ptr(), self.lb, state, self.scr.data_ptr(), self.sb, self.pd,
                                   self.vd, self.w, self.h, self.stream)

    def check(self):
        torch.cuda.synchronize()
        assert allclose_report(self.out.cpu().numpy(), self.d["out"], RTOL, ATOL) <= 1.0
        assert allclose_report(self.wo.cpu().numpy(), self.d["weight"], RTOL, ATOL) <= 1.0
        assert allclose_report(self.gout.cpu().numpy(), self.d["grad_out"], RTOL, ATOL) <= 1.0


def _stats(L):
    c, r = ctypes.c_longlong(0), ctypes.c_longlong(0)
    L.plattice_graph_cache_stats(ctypes.byref(c), ctypes.byref(r))
    return c.value, r.value


@pytest.mark.parametrize("name", ["ref_blobs64_pd5_vd3.npz", "ref_randn24x20_pd16_vd1.npz",
                                  "ref_ragged13x29_pd5_vd3.npz"])
def test_repeated_calls_are_replayed_and_exact(lib, name):
    from plattice_pytorch_b200 import PLOO
    dev = torch.device("cuda:0")
    assert lib.plattice_set_graph_cache(16) == 0
    try:
        b = Buffers(name, dev)
        c0, r0 = _stats(lib)
        for i in range(5):
            b.out.fill_(float("nan"))
            b.gout.fill_(float("nan"))
            assert b.forward(lib) == 0
            assert b.backward(lib, 1) == 0
            b.check()
        c1, r1 = _stats(lib)
        assert c1 - c0 == 2                  # the forward and the backward, captured once each
        assert r1 - r0 == 2 * 3              # calls 3..5 of each replayed the graph call 2 captured
        PLOO.check_device_status()
        # the same calls without graphs give the same result
        assert lib.plattice_set_graph_cache(0) == 0
        b.out.fill_(float("nan"))
        b.gout.fill_(float("nan"))
        assert b.forward(lib) == 0 and b.backward(lib, 1) == 0
        b.check()
        assert _stats(lib)[1] == r1
    finally:
        lib.plattice_set_graph_cache(16)


def test_backward_states_and_other_buffers_get_their_own_graphs(lib):
    dev = torch.device("cuda:0")
    lib.plattice_set_graph_cache(16)
    a = Buffers("ref_blobs64_pd5_vd3.npz", dev)
    b = Buffers("ref_blobs64_pd5_vd3.npz", dev)   # same shapes, other buffers
    for _ in range(3):
        for x in (a, b):
            x.gout.fill_(float("nan"))
            assert x.forward(lib) == 0
            assert x.backward(lib, 1) == 0
            assert x.backward(lib, 2) == 0      # a repeated backward re-zeroes its rows
            assert x.backward(lib, 0) == 0      # a rebuild
            x.check()


def test_device_failure_of_a_replayed_call_is_reported(lib):
    from plattice_pytorch_b200 import PLOO, _lib
    dev = torch.device("cuda:0")
    lib.plattice_set_graph_cache(16)
    PLOO.check_device_status()
    b = Buffers("ref_blobs64_pd5_vd3.npz", dev)
    try:
        lib.plattice_debug_set_table_cap_log2(6)   # 64 cells for 1225 vertices
        c0, r0 = _stats(lib)
        assert b.forward(lib) == 0                 # direct
        torch.cuda.synchronize()
        assert lib.plattice_poll_status() == _lib.ERR_DEVICE
        assert b.forward(lib) == 0                 # captured and launched
        torch.cuda.synchronize()
        assert lib.plattice_poll_status() == _lib.ERR_DEVICE
        assert b.forward(lib) == 0                 # replayed
        torch.cuda.synchronize()
        assert lib.plattice_poll_status() == _lib.ERR_DEVICE
        c1, r1 = _stats(lib)
        assert c1 - c0 == 1 and r1 - r0 == 1
    finally:
        lib.plattice_debug_set_table_cap_log2(0)
    PLOO.check_device_status()
    assert b.forward(lib) == 0 and b.backward(lib, 1) == 0
    b.check()
    torch.cuda.synchronize()
    PLOO.check_device_status()


def test_kept_lattice_filter_loop_replays(lib):
    """Five rounds of filter + filter backward on one kept lattice with fixed
    buffers (a mean-field loop): every round equals the golden forward output,
    normaliser and value gradient; rounds 3..5 replay the captured graphs."""
    from plattice_pytorch_b200 import _lib
    dev = torch.device("cuda:0")
    lib.plattice_set_graph_cache(16)
    b = Buffers("ref_blobs64_pd5_vd3.npz", dev)
    assert b.forward(lib) == 0
    wsb = _lib.filter_workspace_size(b.h, b.w, b.pd, b.vd)
    ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
    c0, r0 = _stats(lib)
    for _ in range(5):
        b.out.fill_(float("nan"))
        b.gout.fill_(float("nan"))
        assert lib.plattice_filter(b.wo.data_ptr(), b.out.data_ptr(), b.v.data_ptr(), b.lat.data_ptr(), b.lb,
                                   ws.data_ptr(), wsb, b.pd, b.vd, b.w, b.h, b.stream) == 0
        assert lib.plattice_filter_backward(b.gout.data_ptr(), b.g.data_ptr(), b.wo.data_ptr(), b.lat.data_ptr(),
                                            b.lb, ws.data_ptr(), wsb, b.pd, b.vd, b.w, b.h, b.stream) == 0
        b.check()
    c1, r1 = _stats(lib)
    assert c1 - c0 == 2 and r1 - r0 == 6


def test_profiling_runs_without_graphs_and_times_groups(lib):
    """Profiling (per launch, or per launch group) runs the calls directly and
    records one interval per launch or per group."""
    from plattice_pytorch_b200 import _lib
    dev = torch.device("cuda:0")
    lib.plattice_set_graph_cache(16)
    b = Buffers("ref_blobs64_pd5_vd3.npz", dev)
    for _ in range(2):   # a graph exists for these buffers from here on
        assert b.forward(lib) == 0 and b.backward(lib, 1) == 0
    _lib.profile_read()
    try:
        c0, r0 = _stats(lib)
        _lib.profile_enable(True)
        assert b.forward(lib) == 0 and b.backward(lib, 1) == 0
        per = _lib.profile_read()
        _lib.profile_enable(True, groups=True)
        assert b.forward(lib) == 0 and b.backward(lib, 1) == 0
        grp = _lib.profile_read()
        assert _stats(lib) == (c0, r0)   # no graph launched while profiling
    finally:
        _lib.profile_enable(False)
    b.check()
    for st in ("tile_build", "clear", "insert", "splat_fwd", "blur_fwd", "slice_fwd", "splat_bwd", "blur_bwd",
               "slice_bwd"):
        assert per[st][1] == 1 and per[st][0] > 0.0, st
    assert all(per[g][1] == 0 for g in ("build", "filter_fwd", "filter_bwd"))
    for g in ("build", "filter_fwd", "filter_bwd"):
        assert grp[g][1] == 1 and grp[g][0] > 0.0, g
    assert all(grp[st][1] == 0 for st in ("tile_build", "splat_fwd", "slice_bwd"))


def test_capture_in_a_torch_cuda_graph(lib):
    """Forward + backward captured by the caller in a torch.cuda.CUDAGraph
    (the library records its launches into the caller's capture, no graph of
    its own) and replayed: the replay on the golden inputs gives the golden
    results, and after new values are copied into the captured input the
    replay equals an eager call on them."""
    from plattice_pytorch_b200 import PLOO
    dev = torch.device("cuda:0")
    lib.plattice_set_graph_cache(16)
    d = np.load(os.path.join(GOLDEN, "ref_blobs64_pd5_vd3.npz"))
    f = torch.from_numpy(d["features"]).to(dev)
    v = torch.from_numpy(d["values"]).to(dev)
    g = torch.from_numpy(d["grad"]).to(dev)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):   # warm-up outside the capture (kernel attributes, lazy loading)
        for _ in range(2):
            wo, out, lat = PLOO.lattice_forward(f, v)
            PLOO.lattice_backward(f, g, wo, lat)
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    cg = torch.cuda.CUDAGraph()
    with torch.cuda.graph(cg):
        wo_c, out_c, lat_c = PLOO.lattice_forward(f, v)
        gr_c = PLOO.lattice_backward(f, g, wo_c, lat_c)
    cg.replay()
    torch.cuda.synchronize()
    assert allclose_report(out_c.cpu().numpy(), d["out"], RTOL, ATOL) <= 1.0
    assert allclose_report(wo_c.cpu().numpy(), d["weight"], RTOL, ATOL) <= 1.0
    assert allclose_report(gr_c.cpu().numpy(), d["grad_out"], RTOL, ATOL) <= 1.0
    v2 = torch.rand_like(v)
    v.copy_(v2)
    cg.replay()
    wo_e, out_e, lat_e = PLOO.lattice_forward(f, v2)
    gr_e = PLOO.lattice_backward(f, g, wo_e, lat_e)
    torch.cuda.synchronize()
    assert allclose_report(out_c.cpu().numpy(), out_e.cpu().numpy(), RTOL, ATOL) <= 1.0
    assert allclose_report(gr_c.cpu().numpy(), gr_e.cpu().numpy(), RTOL, ATOL) <= 1.0
    del cg
    PLOO.check_device_status()


def test_eviction_keeps_results_exact(lib):
    """A cache of two graphs cycled through three sets of buffers: graphs are
    evicted and captured again, and every call still gives the golden result."""
    dev = torch.device("cuda:0")
    assert lib.plattice_set_graph_cache(2) == 0
    try:
        sets = [Buffers("ref_blobs64_pd5_vd3.npz", dev) for _ in range(3)]
        c0, _ = _stats(lib)
        for _ in range(4):
            for b in sets:
                b.out.fill_(float("nan"))
                b.gout.fill_(float("nan"))
                assert b.forward(lib) == 0 and b.backward(lib, 1) == 0
                b.check()
        assert _stats(lib)[0] - c0 >= 4   # more captures than the cache holds: evictions happened
    finally:
        lib.plattice_set_graph_cache(16)


def test_two_host_threads(lib):
    """Two host threads, each with its own buffers and stream, call forward and
    backward concurrently (ctypes releases the GIL during the calls); every
    result equals the golden one."""
    import threading
    dev = torch.device("cuda:0")
    lib.plattice_set_graph_cache(16)
    errors = []

    def worker(name):
        try:
            torch.cuda.set_device(dev)
            s = torch.cuda.Stream(dev)
            with torch.cuda.stream(s):
                b = Buffers(name, dev)
                b.stream = s.cuda_stream
                for _ in range(6):
                    b.out.fill_(float("nan"))
                    b.gout.fill_(float("nan"))
                    assert b.forward(lib) == 0 and b.backward(lib, 1) == 0
                    s.synchronize()
                    assert allclose_report(b.out.cpu().numpy(), b.d["out"], RTOL, ATOL) <= 1.0
                    assert allclose_report(b.gout.cpu().numpy(), b.d["grad_out"], RTOL, ATOL) <= 1.0
        except BaseException as e:   # reported by the main thread
            errors.append(repr(e))

    threads = [threading.Thread(target=worker, args=(n,))
               for n in ("ref_blobs64_pd5_vd3.npz", "ref_randn24x20_pd16_vd1.npz")]
    for th in threads:
        th.start()
    for th in threads:
        th.join(timeout=120)
    assert not any(th.is_alive() for th in threads)
    assert not errors, errors
