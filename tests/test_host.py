"""Host-side checks that need no GPU: the C ABI library loads and exports every
function include/plattice.h declares, its argument checks, the Python layer's
input checks (the reference's messages), and the multi-rank plumbing over gloo."""
import ctypes
import os
import re
import socket

import numpy as np
import pytest
import torch

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "plattice.h")


def _declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(plattice_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from plattice_pytorch_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        pytest.skip("libplattice_b200.so not built (python -m plattice_pytorch_b200.build)")
    return _lib.lib()


def test_every_declared_symbol_is_exported(lib):
    names = _declared_functions()
    assert len(names) >= 10
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_abi_version_and_error_strings(lib):
    from plattice_pytorch_b200 import _lib
    assert lib.plattice_abi_version() == _lib.ABI_VERSION
    for code in range(5):
        assert _lib.error_string(code)


def test_workspace_sizes_and_argument_checks(lib):
    from plattice_pytorch_b200 import _lib
    lb, sb = _lib.workspace_sizes(1024, 1024, 5, 3)
    assert lb > 1024 * 1024 * 6 * 6 and sb > 0
    lb0, sb0 = _lib.workspace_sizes(0, 7, 5, 3)
    assert lb0 == 256 and sb0 == 256
    for pd, vd in [(0, 3), (17, 3), (5, 0), (5, 9)]:
        with pytest.raises(_lib.PlatticeError):
            _lib.workspace_sizes(8, 8, pd, vd)
    # invalid dimensions are refused before anything touches a device
    S = ctypes.c_size_t
    lib.plattice_forward.argtypes = [ctypes.c_void_p] * 5 + [S, ctypes.c_void_p, S] + [ctypes.c_int] * 4 + [ctypes.c_void_p]
    assert lib.plattice_forward(None, None, None, None, None, 0, None, 0, 0, 3, 8, 8, None) == _lib.ERR_INVALID
    assert lib.plattice_forward(None, None, None, None, None, 0, None, 0, 5, 3, 8, 8, None) == _lib.ERR_INVALID


def test_kept_lattice_sizes_and_argument_checks(lib):
    """plattice_filter / plattice_filter_backward refuse bad arguments and
    undersized buffers before any CUDA call."""
    from plattice_pytorch_b200 import _lib
    b = _lib.filter_workspace_size(1024, 1024, 5, 3)
    lb, _ = _lib.workspace_sizes(1024, 1024, 5, 3)
    assert b >= 2 * 1024 * 1024 * 6 * 4 * 4   # two value-row buffers of slots x 4 floats
    assert _lib.filter_workspace_size(0, 5, 5, 3) == 256
    for pd, vd in [(0, 3), (17, 3), (5, 0), (5, 9)]:
        with pytest.raises(_lib.PlatticeError):
            _lib.filter_workspace_size(8, 8, pd, vd)
    fake = ctypes.c_void_p(256)   # never dereferenced: every call below returns before using it
    # invalid dimensions, missing pointers
    assert lib.plattice_filter(fake, fake, fake, fake, lb, fake, b, 0, 3, 8, 8, None) == _lib.ERR_INVALID
    assert lib.plattice_filter(None, fake, fake, fake, lb, fake, b, 5, 3, 8, 8, None) == _lib.ERR_INVALID
    assert lib.plattice_filter_backward(fake, fake, None, fake, lb, fake, b, 5, 3, 8, 8, None) == _lib.ERR_INVALID
    # undersized lattice or value workspace
    lb8, _ = _lib.workspace_sizes(8, 8, 5, 3)
    b8 = _lib.filter_workspace_size(8, 8, 5, 3)
    assert lib.plattice_filter(fake, fake, fake, fake, 1000, fake, b8, 5, 3, 8, 8, None) == _lib.ERR_WORKSPACE
    assert lib.plattice_filter(fake, fake, fake, fake, lb8, fake, b8 - 1, 5, 3, 8, 8, None) == _lib.ERR_WORKSPACE
    assert lib.plattice_filter_backward(fake, fake, fake, fake, lb8, fake, 16, 5, 3, 8, 8, None) == _lib.ERR_WORKSPACE
    # a rebuild needs the features
    assert lib.plattice_backward(fake, fake, fake, None, fake, lb8, 0, fake, 1 << 30, 5, 3, 8, 8,
                                 None) == _lib.ERR_INVALID
    # every backward needs a scratch: the full one for a rebuild, the front part otherwise
    rb8 = _lib.reuse_scratch_size(1, 8, 8, 5, 3)
    _, sb8 = _lib.workspace_sizes(8, 8, 5, 3)
    assert rb8 < sb8
    assert lib.plattice_backward(fake, fake, fake, None, fake, lb8, 1, None, 0, 5, 3, 8, 8,
                                 None) == _lib.ERR_INVALID
    assert lib.plattice_backward(fake, fake, fake, None, fake, lb8, 1, fake, rb8 - 1, 5, 3, 8, 8,
                                 None) == _lib.ERR_WORKSPACE
    assert lib.plattice_backward(fake, fake, fake, fake, fake, lb8, 0, fake, rb8, 5, 3, 8, 8,
                                 None) == _lib.ERR_WORKSPACE
    # only the lattice's last array (the first backward's rows) depends on vd:
    # a filter accepts a lattice built with a smaller vd
    assert _lib.workspace_sizes(8, 8, 5, 1)[0] < lb8 < _lib.workspace_sizes(8, 8, 5, 8)[0]


def test_batch_sizes_and_argument_checks(lib):
    from plattice_pytorch_b200 import _lib
    lb, sb = _lib.workspace_sizes(512, 512, 5, 3)
    blb, bsb = _lib.batch_workspace_sizes(64, 512, 512, 5, 3)
    # one lattice for the batch: every array scales with the images, only the
    # header and the 256-byte padding of each array do not
    assert 64 * lb - 64 * 4096 <= blb <= 64 * lb
    assert bsb >= 64 * _lib.reuse_scratch_size(1, 512, 512, 5, 3)
    assert _lib.reuse_scratch_size(64, 512, 512, 5, 3) < bsb
    with pytest.raises(_lib.PlatticeError):
        _lib.batch_workspace_sizes(-1, 8, 8, 5, 3)
    fake = ctypes.c_void_p(256)
    assert lib.plattice_forward_batch(fake, fake, fake, fake, fake, blb, fake, bsb, -2, 5, 3, 8, 8,
                                      None) == _lib.ERR_INVALID
    assert lib.plattice_forward_batch(fake, fake, fake, fake, fake, blb, fake, bsb, 3, 0, 3, 8, 8,
                                      None) == _lib.ERR_INVALID
    lb8, sb8 = _lib.batch_workspace_sizes(3, 8, 8, 5, 3)
    assert lib.plattice_forward_batch(fake, fake, fake, fake, fake, lb8 - 1, fake, sb8, 3, 5, 3, 8, 8,
                                      None) == _lib.ERR_WORKSPACE
    assert lib.plattice_backward_batch(fake, fake, fake, None, fake, lb8, 0, fake, sb8, 3, 5, 3, 8, 8,
                                       None) == _lib.ERR_INVALID
    assert lib.plattice_forward_batch(None, None, None, None, None, 0, None, 0, 0, 5, 3, 8, 8,
                                      None) == _lib.OK   # an empty batch is a no-op


def test_feature_grad_sizes_and_argument_checks(lib):
    from plattice_pytorch_b200 import _lib
    b = _lib.feature_grad_workspace_size(512, 512, 5, 3)
    slots = 512 * 512 * 6   # tiles x K x P for a 512 x 512 image at pd 5
    assert b >= 4 * slots * 4 * 4 + 512 * 512 * 4 * 4   # R and H ping-pong rows + (G, -G.out) rows
    with pytest.raises(_lib.PlatticeError):
        _lib.feature_grad_workspace_size(8, 8, 17, 3)
    fake = ctypes.c_void_p(256)
    lb8, _ = _lib.workspace_sizes(8, 8, 5, 3)
    b8 = _lib.feature_grad_workspace_size(8, 8, 5, 3)
    args = [fake] * 7 + [lb8, fake, b8, 5, 3, 8, 8, None]
    bad = list(args); bad[5] = None   # no features
    assert lib.plattice_feature_grad(*bad) == _lib.ERR_INVALID
    small = list(args); small[9] = b8 - 1
    assert lib.plattice_feature_grad(*small) == _lib.ERR_WORKSPACE
    small = list(args); small[7] = 100
    assert lib.plattice_feature_grad(*small) == _lib.ERR_WORKSPACE


def test_lattice_precision_setting(lib):
    """Host side of the reduced-precision lattice values: only 32 and 16 bits
    are accepted, the setting reads back, and the Python wrapper checks its
    argument (no GPU call)."""
    from plattice_pytorch_b200 import PLOO
    from plattice_pytorch_b200 import _lib
    try:
        assert lib.plattice_get_lattice_precision() == 32
        assert lib.plattice_set_lattice_precision(8) == _lib.ERR_INVALID
        assert lib.plattice_get_lattice_precision() == 32
        assert lib.plattice_set_lattice_precision(16) == _lib.OK
        assert PLOO.get_lattice_precision() == "bf16"
        PLOO.set_lattice_precision("fp32")
        assert lib.plattice_get_lattice_precision() == 32
        with pytest.raises(RuntimeError, match="lattice precision"):
            PLOO.set_lattice_precision("fp16")
    finally:
        lib.plattice_set_lattice_precision(32)


def test_python_checks_raise_reference_messages():
    from plattice_pytorch_b200 import PLOO
    f = torch.zeros(4, 4, 5)
    v = torch.zeros(4, 4, 3)
    with pytest.raises(RuntimeError, match="features must be CUDA"):
        PLOO.forward(f, v)
    with pytest.raises(RuntimeError, match="features must be CUDA"):
        PLOO.backward(f, v, torch.zeros(4, 4, 1))
    with pytest.raises(RuntimeError, match="lattice must be a Lattice"):
        PLOO.lattice_filter(object(), v)
    with pytest.raises(RuntimeError, match="features must be CUDA"):
        PLOO.forward_batch(torch.zeros(2, 4, 4, 5), torch.zeros(2, 4, 4, 3))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import torch.distributed as dist
    from plattice_pytorch_b200.sharding import barrier, max_over_ranks, shard_range
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        start, stop = shard_range(64, world, rank)
        barrier(world)
        mx = max_over_ranks(10.0 + rank, world)
        q.put((rank, start, stop, mx))
    finally:
        dist.destroy_process_group()


def test_image_sharding_over_two_gloo_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [(r[1], r[2]) for r in res] == [(0, 32), (32, 64)]
    assert all(r[3] == 11.0 for r in res)


def test_shard_range_partitions_any_batch():
    from plattice_pytorch_b200.sharding import shard_range
    for n in (0, 1, 7, 64, 65):
        for world in (1, 2, 3, 8):
            parts = [shard_range(n, world, r) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
            assert max(p[1] - p[0] for p in parts) - min(p[1] - p[0] for p in parts) <= 1


def test_cpp_function_extension_loads_and_checks_inputs(lib):
    """The C++ build of PermutoLatticeFunction (extension _plattice_torch) loads,
    takes the library's entry points, and rejects bad inputs with the
    reference's messages before any device work (CPU tensors here)."""
    from plattice_pytorch_b200 import plattice
    if not os.path.exists(os.path.join(ROOT, "plattice_pytorch_b200", "_plattice_torch.so")):
        pytest.skip("_plattice_torch.so not built (python -m plattice_pytorch_b200.build)")
    fn = plattice._cpp_function()
    assert fn is not None
    with pytest.raises(RuntimeError, match="features must be CUDA"):
        fn(torch.zeros(4, 4, 5), torch.zeros(4, 4, 3))
    with pytest.raises(RuntimeError, match="features must be CUDA"):
        plattice.PermutoLatticeFunction.apply(torch.zeros(4, 4, 5), torch.zeros(4, 4, 3))


def test_a_broken_lattice_no_longer_matches_and_is_refused():
    """Host logic of a lattice after a failed call on it (CPU tensors stand in
    for the device buffers; no library call): it stops matching its features,
    so a backward rebuilds, and the kept-lattice calls refuse it."""
    from plattice_pytorch_b200 import PLOO
    f = torch.zeros(4, 5, 3)
    lat = PLOO.Lattice(f, 2, torch.empty(16, dtype=torch.uint8), None)
    assert lat.matches(f, 2) and not lat.broken
    lat.broken = True
    assert not lat.matches(f, 2) and not lat.matches(f, 2, same_object=False)
    with pytest.raises(RuntimeError, match="unusable"):
        PLOO._check_kept(lat, torch.zeros(4, 5, 2), "values")
    fb = torch.zeros(2, 4, 5, 3)
    b = PLOO.BatchLattice(fb, 2, torch.empty(16, dtype=torch.uint8))
    assert b.matches(fb, 2)
    b.broken = True
    assert not b.matches(fb, 2)
