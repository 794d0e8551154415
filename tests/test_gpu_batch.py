"""Batches of images in one call (``PLOO.forward_batch`` / ``backward_batch``,
C ABI ``plattice_forward_batch`` / ``plattice_backward_batch``).

The reference filters one image per call (its callers loop over a batch in
Python), so the checker is the single-image path on every image of the batch,
which the other GPU tests pin to the reference: outputs, normalisers and
value gradients of the batch call equal the per-image calls within 1e-5
relative + 5e-6 absolute (float reductions in another order); the batch
backward reuses the batch's lattices or rebuilds them; autograd through
``PermutoLatticeBatchFunction`` equals autograd through
``PermutoLatticeFunction`` image by image.
"""
import numpy as np
import pytest
import torch

from conftest import allclose_report

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 5e-6


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from plattice_pytorch_b200 import _lib
    _lib.lib()
    return torch.device("cuda:0")


def _close(a, b):
    return allclose_report(a.detach().cpu().numpy(), b.detach().cpu().numpy(), RTOL, ATOL) <= 1.0


def _batch(name, b, dev):
    from plattice_pytorch_b200.workloads import make_workload
    ws = [make_workload(name, seed=5 + i, index=i) for i in range(b)]
    st = lambda k: torch.from_numpy(np.stack([w[k] for w in ws])).to(dev).contiguous()
    return st("features"), st("values"), st("grad")


@pytest.mark.parametrize("name,b", [("blobs64_pd5_vd3", 3), ("crf512_pd5_vd3", 2), ("blobs64_pd5_vd3", 1)])
def test_batch_equals_the_images_one_by_one(name, b, dev):
    from plattice_pytorch_b200 import PLOO
    f, v, g = _batch(name, b, dev)
    wb, ob = PLOO.forward_batch(f, v)
    gb = PLOO.backward_batch(f, g, wb)            # reuses the batch's lattices
    gb2 = PLOO.batch_backward(f, g, wb, None)     # rebuilds them
    for i in range(b):
        wi, oi = PLOO.forward(f[i], v[i])
        gi = PLOO.backward(f[i], g[i], wi)
        assert _close(ob[i], oi) and _close(wb[i], wi)
        assert _close(gb[i], gi) and _close(gb2[i], gi)


def test_batch_with_odd_shape_and_pd16(dev):
    from plattice_pytorch_b200 import PLOO
    gen = torch.Generator().manual_seed(3)
    f = (torch.randn((3, 13, 29, 16), generator=gen) * 2).to(dev)
    v = torch.rand((3, 13, 29, 2), generator=gen).to(dev)
    wb, ob = PLOO.forward_batch(f, v)
    for i in range(3):
        wi, oi = PLOO.forward(f[i].contiguous(), v[i].contiguous())
        assert _close(ob[i], oi) and _close(wb[i], wi)


def test_autograd_through_the_batch(dev):
    from plattice_pytorch_b200 import PermutoLatticeBatchFunction, PermutoLatticeFunction
    f, v, g = _batch("blobs64_pd5_vd3", 2, dev)
    a = v.clone().requires_grad_(True)
    ob = PermutoLatticeBatchFunction.apply(f, a)
    (ga,) = torch.autograd.grad(ob, (a,), (g,))
    for i in range(2):
        b = v[i].clone().requires_grad_(True)
        oi = PermutoLatticeFunction.apply(f[i], b)
        (gi,) = torch.autograd.grad(oi, (b,), (g[i],))
        assert _close(ob[i], oi) and _close(ga[i], gi)


def test_batch_checks_shapes(dev):
    from plattice_pytorch_b200 import PLOO
    f, v, _ = _batch("blobs64_pd5_vd3", 2, dev)
    with pytest.raises(RuntimeError, match="matching B, H, W"):
        PLOO.forward_batch(f, v[:1])
    with pytest.raises(RuntimeError, match=r"features must be \[B, H, W, pd\]"):
        PLOO.forward_batch(f[0], v)


def test_batch_images_against_golden_and_oracle(dev):
    """Images of a batch against checkers outside this library: the golden
    vectors the reference CUDA build produced for one image, placed first and
    last in a batch, and the CPU oracle for the image between them; the
    batch's vertex count is the sum of the images' own (equal keys of
    different images stay different vertices)."""
    import os
    import oracle
    from conftest import GOLDEN
    from plattice_pytorch_b200 import PLOO
    from plattice_pytorch_b200.workloads import make_workload
    d = np.load(os.path.join(GOLDEN, "ref_blobs64_pd5_vd3.npz"))
    other = make_workload("blobs64_pd5_vd3", seed=9)
    f = torch.from_numpy(np.stack([d["features"], other["features"], d["features"]])).to(dev)
    v = torch.from_numpy(np.stack([d["values"], other["values"], d["values"]])).to(dev)
    g = torch.from_numpy(np.stack([d["grad"], other["grad"], d["grad"]])).to(dev)
    wb, ob, lat = PLOO.batch_forward(f, v)
    gb = PLOO.batch_backward(f, g, wb, lat)
    m_other = oracle.vertex_keys(other["features"])[0].shape[0]
    assert PLOO.lattice_info(lat)["m"] == 2 * int(d["m"]) + m_other
    for i in (0, 2):
        assert allclose_report(ob[i].cpu().numpy(), d["out"], RTOL, ATOL) <= 1.0
        assert allclose_report(wb[i].cpu().numpy(), d["weight"], RTOL, ATOL) <= 1.0
        assert allclose_report(gb[i].cpu().numpy(), d["grad_out"], RTOL, ATOL) <= 1.0
    wo, out, _ = oracle.forward(other["features"], other["values"])
    assert allclose_report(ob[1].cpu().numpy(), out, RTOL, ATOL) <= 1.0
    assert allclose_report(wb[1].cpu().numpy(), wo, RTOL, ATOL) <= 1.0
    go = oracle.backward(other["features"], other["grad"], wb[1].cpu().numpy())
    assert allclose_report(gb[1].cpu().numpy(), go, RTOL, ATOL) <= 1.0


def test_full_size_batch_vs_reference_cuda(dev):
    """Three 512x512 dense-CRF images in one batch call against the reference
    CUDA build run on each image (skipped when oracle/_ref was not built)."""
    from oracle import ref as oref
    if not oref.available():
        pytest.skip("reference build (oracle/_ref) not present")
    from plattice_pytorch_b200 import PLOO
    f, v, g = _batch("crf512_pd5_vd3", 3, dev)
    wb, ob, lat = PLOO.batch_forward(f, v)
    R = oref.RefLattice()
    m_total, w_ref = 0, []
    for i in range(3):
        wo_r, out_r, ws = R.forward(f[i].contiguous(), v[i].contiguous())
        m_total += R.lattice(ws, f.shape[1] * f.shape[2], f.shape[3])["m"]
        del ws
        assert allclose_report(ob[i].cpu().numpy(), out_r.cpu().numpy(), RTOL, ATOL) <= 1.0
        assert allclose_report(wb[i].cpu().numpy(), wo_r.cpu().numpy(), RTOL, ATOL) <= 1.0
        w_ref.append(wo_r)
    assert PLOO.lattice_info(lat)["m"] == m_total
    # both backward passes from the reference's normalisers, so that the
    # gradient comparison isolates the backward
    gb = PLOO.batch_backward(f, g, torch.stack(w_ref).contiguous(), lat)
    for i in range(3):
        grad_r = R.backward(f[i].contiguous(), g[i].contiguous(), w_ref[i])
        assert allclose_report(gb[i].cpu().numpy(), grad_r.cpu().numpy(), RTOL, ATOL) <= 1.0
