"""Generate the golden fixtures under tests/golden/.

Two sources, two modes:

``python tests/golden/make_golden.py image --ref <reference tree>``
    Runs where the reference tree is mounted (CPU is enough).  Takes the
    32x32 crop [48:80, 48:80] of the reference test image
    (tests/assets/test_image.png), builds its features with the reference
    test's recipe and computes the reference's own brute_force_bilateral
    (tests/test_plattice.py:58-77) by importing the reference test module.
    Writes bilateral_crop.npz (crop, features, brute-force output).

``python tests/golden/make_golden.py reference --out DIR [--big]``
    Runs on a GPU with the reference CUDA filter prebuilt in oracle/_ref
    (``make -C oracle ref``).  For every case below it runs the reference
    forward and backward on seeded inputs and records the inputs, the lattice
    the reference built (sorted vertex key set, per-slot vertex index into
    it, per-slot barycentric weights) and the outputs.  Writes
    DIR/ref_<case>.npz.  ``--big`` adds larger cases used to pin the oracle's
    float contraction variant (not committed: too large).
"""
import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)


def small_cases():
    """name -> dict(features, values, grad); all seeded."""
    from plattice_pytorch_b200.workloads import make_workload
    cases = {}
    cases["blobs64_pd5_vd3"] = make_workload("blobs64_pd5_vd3")
    rng = np.random.default_rng(7)
    f = rng.standard_normal((16, 16, 5)).astype(np.float32)
    v = rng.standard_normal((16, 16, 3)).astype(np.float32)
    cases["randn16_pd5_vd3"] = {"features": f, "values": v, "grad": np.ones_like(v)}
    rng = np.random.default_rng(11)
    for pd, vd in [(1, 1), (2, 4), (5, 3), (8, 2)]:
        f = rng.standard_normal((12, 10, pd)).astype(np.float32)
        v = rng.standard_normal((12, 10, vd)).astype(np.float32)
        cases[f"randn12x10_pd{pd}_vd{vd}"] = {"features": f, "values": v, "grad": np.ones_like(v)}
    rng = np.random.default_rng(23)
    for pd in range(1, 17):
        vd = (pd % 8) + 1
        f = (rng.standard_normal((24, 20, pd)) * 1.5).astype(np.float32)
        v = rng.uniform(-1, 1, (24, 20, vd)).astype(np.float32)
        g = rng.standard_normal((24, 20, vd)).astype(np.float32)
        cases[f"randn24x20_pd{pd}_vd{vd}"] = {"features": f, "values": v, "grad": g}
    # pd 16 stress at a fixture-friendly size
    rng = np.random.default_rng(4)
    f = (rng.standard_normal((16, 16, 16)) * 2.0).astype(np.float32)
    v = rng.uniform(-1, 1, (16, 16, 8)).astype(np.float32)
    cases["gauss16_pd16_vd8"] = {"features": f, "values": v,
                                 "grad": rng.standard_normal((16, 16, 8)).astype(np.float32)}
    # every pixel in one simplex
    rng = np.random.default_rng(5)
    f = np.empty((64, 64, 2), np.float32)
    f[..., 0], f[..., 1] = 0.3, 0.7
    v = rng.uniform(-1, 1, (64, 64, 8)).astype(np.float32)
    cases["collapse64_pd2_vd8"] = {"features": f, "values": v,
                                   "grad": rng.standard_normal((64, 64, 8)).astype(np.float32)}
    # quantised features: exact ties in the greedy rounding and in the rank sort
    rng = np.random.default_rng(31)
    for pd, q in [(5, 4.0), (3, 2.0), (2, 1.0)]:
        f = (rng.integers(-24, 25, (40, 40, pd)) / q).astype(np.float32)
        v = rng.uniform(0, 1, (40, 40, 3)).astype(np.float32)
        cases[f"quant40_pd{pd}_vd3"] = {"features": f, "values": v,
                                        "grad": rng.standard_normal((40, 40, 3)).astype(np.float32)}
    # empty-ish and ragged shapes
    rng = np.random.default_rng(37)
    for (h, w) in [(1, 1), (1, 7), (9, 1), (13, 29)]:
        f = rng.standard_normal((h, w, 5)).astype(np.float32)
        v = rng.standard_normal((h, w, 3)).astype(np.float32)
        cases[f"ragged{h}x{w}_pd5_vd3"] = {"features": f, "values": v,
                                          "grad": rng.standard_normal((h, w, 3)).astype(np.float32)}
    return cases


def big_cases():
    from plattice_pytorch_b200.workloads import make_workload
    cases = {"blobs256_pd5_vd3": make_workload("blobs256_pd5_vd3"),
             "crf512_pd5_vd3_i1": make_workload("crf512_pd5_vd3", index=1)}
    rng = np.random.default_rng(4)
    f = (rng.standard_normal((128, 128, 16)) * 2.0).astype(np.float32)
    v = rng.uniform(-1, 1, (128, 128, 8)).astype(np.float32)
    cases["gauss128_pd16_vd8"] = {"features": f, "values": v,
                                  "grad": rng.standard_normal((128, 128, 8)).astype(np.float32)}
    return cases


def lattice_record(slot_keys, slot_w):
    """Sorted vertex key set plus, per slot, the index of its key in that set."""
    n, K, pd = slot_keys.shape
    flat = slot_keys.reshape(n * K, pd)
    vkeys, inv = np.unique(flat, axis=0, return_inverse=True)
    return vkeys.astype(np.int16), inv.reshape(n, K).astype(np.int32), slot_w.astype(np.float32)


def run_reference(out_dir, big):
    import torch
    from oracle.ref import RefLattice
    ref = RefLattice()
    dev = torch.device("cuda:0")
    cases = small_cases()
    if big:
        cases.update(big_cases())
    os.makedirs(out_dir, exist_ok=True)
    for name, c in cases.items():
        f = torch.from_numpy(c["features"]).to(dev).contiguous()
        v = torch.from_numpy(c["values"]).to(dev).contiguous()
        g = torch.from_numpy(c["grad"]).to(dev).contiguous()
        h, w, pd = f.shape
        wo, out, ws = ref.forward(f, v)
        lat = ref.lattice(ws, h * w, pd)
        gout = ref.backward(f, g, wo)
        vkeys, slot_vertex, slot_w = lattice_record(lat["slot_keys"], lat["slot_w"])
        if vkeys.shape[0] != lat["m"]:
            print(f"{name}: note: distinct slot keys {vkeys.shape[0]} != canonical slots {lat['m']}")
        np.savez_compressed(
            os.path.join(out_dir, f"ref_{name}.npz"),
            features=c["features"], values=c["values"], grad=c["grad"],
            vertex_keys=vkeys, slot_vertex=slot_vertex, slot_w=slot_w, m=np.int64(lat["m"]),
            weight=wo.cpu().numpy(), out=out.cpu().numpy(), grad_out=gout.cpu().numpy())
        print(f"{name}: m={lat['m']} out[{out.min().item():.4g},{out.max().item():.4g}]", flush=True)


def run_image(out_dir, ref_root):
    import importlib.util
    from PIL import Image
    spec = importlib.util.spec_from_file_location(
        "ref_test_plattice", os.path.join(ref_root, "tests", "test_plattice.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    image = np.asarray(Image.open(os.path.join(ref_root, "tests", "assets", "test_image.png"))
                       .convert("RGB"), dtype=np.float32) / 255.0
    crop = image[48:80, 48:80].copy()
    feats = mod.make_features(crop)
    brute = mod.brute_force_bilateral(crop)
    np.savez_compressed(os.path.join(out_dir, "bilateral_crop.npz"), crop=crop.astype(np.float32),
                        features=feats.astype(np.float32), brute=brute.astype(np.float32),
                        sigma_s=np.float32(8.0), sigma_r=np.float32(0.1),
                        psnr_floor=np.float32(18.0))
    print("bilateral_crop.npz written", crop.shape, float(brute.min()), float(brute.max()))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("mode", choices=["image", "reference"])
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--big", action="store_true")
    ap.add_argument("--ref", help="the reference source tree (mode image: its test module and test image)")
    a = ap.parse_args()
    if a.mode == "image":
        if not a.ref:
            ap.error("mode image reads the reference's test files: pass --ref <reference tree>")
        run_image(a.out, a.ref)
    else:
        run_reference(a.out, a.big)


if __name__ == "__main__":
    main()
