"""Device memory of the filter on the headline image (1024 x 1024, pd 5, vd 3),
measured with PyTorch's allocator counters around the public calls.

What a forward keeps for its backward is the lattice buffer alone (per-slot
records, staged vertex ids, blur neighbours, the first backward's value rows);
the build's scratch -- staged keys, hash table, vertex keys, forward value
rows -- is returned when the forward returns, and a backward that reuses the
lattice takes only one value-row buffer and the blur's bookkeeping.  The
buffers are sized for the worst case (every slot a distinct vertex) because
the vertex count is known only on the device and no call synchronises.

Ceilings: retained <= 500 MiB (590 MiB before the backward's value rows and
the blur bookkeeping moved out of the kept lattice), forward peak <= 1.05 GiB,
backward transient <= 128 MiB.  The reference keeps nothing but allocates its
whole workspace (636 MiB at vd 4) in the forward and again in the backward
(permuto.cpp:42-69).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

MiB = 1 << 20


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from plattice_pytorch_b200 import _lib
    _lib.lib()
    return torch.device("cuda:0")


def test_retained_and_peak_bytes(dev):
    from plattice_pytorch_b200 import PLOO, _lib
    from plattice_pytorch_b200.workloads import make_workload
    w = make_workload("voronoi1024_pd5_vd3")
    f = torch.from_numpy(w["features"]).to(dev)
    v = torch.from_numpy(w["values"]).to(dev)
    g = torch.from_numpy(w["grad"]).to(dev)
    h, wd, pd = f.shape
    vd = v.shape[2]
    lb, sb = _lib.workspace_sizes(h, wd, pd, vd)
    rb = _lib.reuse_scratch_size(1, h, wd, pd, vd)
    outputs = h * wd * (vd + 1) * 4

    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats(dev)
    base = torch.cuda.memory_allocated(dev)
    weight, out, lat = PLOO.lattice_forward(f, v)
    torch.cuda.synchronize()
    fwd_peak = torch.cuda.max_memory_allocated(dev) - base
    retained = torch.cuda.memory_allocated(dev) - base - outputs
    assert lb <= retained <= lb + 2 * MiB
    assert retained <= 500 * MiB
    assert fwd_peak <= lb + sb + outputs + 4 * MiB
    assert fwd_peak <= 1075 * MiB

    torch.cuda.reset_peak_memory_stats(dev)
    before = torch.cuda.memory_allocated(dev)
    grad = PLOO.lattice_backward(f, g, weight, lat)
    torch.cuda.synchronize()
    bwd_transient = torch.cuda.max_memory_allocated(dev) - before - grad.numel() * 4
    assert bwd_transient <= rb + 2 * MiB
    assert bwd_transient <= 128 * MiB
    assert PLOO.lattice_info(lat)["status"] == 0
    assert np.isfinite(grad.cpu().numpy()).all()
