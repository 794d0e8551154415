"""Seeded synthetic inputs for the permutohedral-lattice filter.

Every workload is a dict of float32 numpy arrays ``features [H,W,pd]``,
``values [H,W,vd]`` and ``grad [H,W,vd]`` (the upstream gradient), generated
from a seed so that the tests, the golden-vector script and the benchmark all
see the same data.  No dataset is involved: the images are synthetic.

Named workloads (name -> what it is):

* ``blobs64_pd5_vd3``      64x64 RGB image of 8 alpha-composited Gaussian blobs plus
  uniform noise of amplitude 0.02, clipped to [0,1]; features (x/8, y/8, rgb/0.125);
  values = rgb.  Small enough for the brute-force Gaussian.
* ``blobs256_pd5_vd3``     256x256, 64 blobs; features (x/16, y/16, rgb/0.1); values = rgb.
* ``voronoi1024_pd5_vd4``  1024x1024 image of 200 Voronoi cells, each a random colour
  plus a linear gradient, plus N(0, 0.03^2) noise; features (x/32, y/32, rgb/0.08);
  values (r, g, b, 1).
* ``voronoi1024_pd5_vd3``  the same image with values = rgb (the headline throughput case).
* ``gauss512_pd16_vd8``    512x512, features i.i.d. N(0,1)*2 (pd 16), values U(-1,1) (vd 8).
* ``gauss256_pd16_vd8``    the same distribution at 256x256 (1.1 M lattice vertices): a
  case small enough for full profiler captures of the large-lattice kernels.
* ``collapse512_pd2_vd8``  512x512, every feature vector (0.3, 0.7) so every pixel falls
  in one simplex (pd+1 = 3 lattice vertices), values U(-1,1) (vd 8).
* ``crf512_pd5_vd3``       one image of a batch of 512x512 images (``index`` selects it;
  even indices blobs, odd Voronoi, seed = base seed + index); features
  (x/20, y/20, rgb/0.1); values a 3-class softmax of N(0,1) logits.
"""
import numpy as np

__all__ = ["WORKLOADS", "make_workload", "blob_image", "voronoi_image", "spatial_rgb_features"]


def blob_image(h, w, n_blobs, seed, noise=0.02):
    """Alpha-composite ``n_blobs`` Gaussian blobs of random colour over a random
    background, add U(-noise, noise) and clip to [0, 1]."""
    rng = np.random.default_rng(seed)
    ys, xs = np.meshgrid(np.arange(h, dtype=np.float32), np.arange(w, dtype=np.float32),
                         indexing="ij")
    img = np.empty((h, w, 3), np.float32)
    img[:] = rng.uniform(0.0, 1.0, 3).astype(np.float32)
    size = float(min(h, w))
    for _ in range(n_blobs):
        cx, cy = rng.uniform(0, w), rng.uniform(0, h)
        s = rng.uniform(0.04, 0.2) * size
        col = rng.uniform(0.0, 1.0, 3).astype(np.float32)
        a = np.exp(-((xs - cx) ** 2 + (ys - cy) ** 2) / np.float32(2.0 * s * s)).astype(np.float32)
        img = img * (1.0 - a[..., None]) + a[..., None] * col
    img += rng.uniform(-noise, noise, img.shape).astype(np.float32)
    return np.clip(img, 0.0, 1.0).astype(np.float32)


def voronoi_image(h, w, n_cells, seed, noise_sigma=0.03):
    """Piecewise-smooth image: ``n_cells`` Voronoi cells, each a random colour plus a
    random linear gradient (clipped to [0,1]), plus N(0, noise_sigma^2) noise."""
    rng = np.random.default_rng(seed)
    sx = rng.uniform(0, w, n_cells).astype(np.float32)
    sy = rng.uniform(0, h, n_cells).astype(np.float32)
    base = rng.uniform(0.0, 1.0, (n_cells, 3)).astype(np.float32)
    grad = rng.uniform(-0.5, 0.5, (n_cells, 3, 2)).astype(np.float32)
    img = np.empty((h, w, 3), np.float32)
    xs = np.arange(w, dtype=np.float32)
    rows = max(1, (1 << 22) // max(1, w * n_cells))
    for y0 in range(0, h, rows):
        y1 = min(h, y0 + rows)
        ys = np.arange(y0, y1, dtype=np.float32)
        d2 = (xs[None, :, None] - sx) ** 2 + (ys[:, None, None] - sy) ** 2
        cell = np.argmin(d2, axis=-1)
        dx = (xs[None, :] - sx[cell]) / np.float32(w)
        dy = (ys[:, None] - sy[cell]) / np.float32(h)
        img[y0:y1] = base[cell] + grad[cell, :, 0] * dx[..., None] + grad[cell, :, 1] * dy[..., None]
    img = np.clip(img, 0.0, 1.0)
    img += rng.normal(0.0, noise_sigma, img.shape).astype(np.float32)
    return img.astype(np.float32)


def spatial_rgb_features(img, sigma_s, sigma_r):
    """(x/sigma_s, y/sigma_s, r/sigma_r, g/sigma_r, b/sigma_r), the feature layout of
    the reference test (tests/test_plattice.py:39-55)."""
    h, w, _ = img.shape
    ys, xs = np.meshgrid(np.arange(h, dtype=np.float32), np.arange(w, dtype=np.float32),
                         indexing="ij")
    return np.concatenate(
        [xs[..., None] / np.float32(sigma_s), ys[..., None] / np.float32(sigma_s),
         img / np.float32(sigma_r)], axis=-1).astype(np.float32)


def _grad(rng, shape):
    return rng.standard_normal(shape).astype(np.float32)


def _softmax3(rng, h, w):
    z = rng.standard_normal((h, w, 3)).astype(np.float32)
    z = np.exp(z - z.max(axis=-1, keepdims=True))
    return (z / z.sum(axis=-1, keepdims=True)).astype(np.float32)


def make_workload(name, seed=0, index=0):
    """Return ``dict(features, values, grad)`` for a named workload (see module doc)."""
    s = 1000003 * seed
    if name == "blobs64_pd5_vd3":
        img = blob_image(64, 64, 8, s + 1)
        f, v = spatial_rgb_features(img, 8.0, 0.125), img
    elif name == "blobs256_pd5_vd3":
        img = blob_image(256, 256, 64, s + 2)
        f, v = spatial_rgb_features(img, 16.0, 0.1), img
    elif name in ("voronoi1024_pd5_vd4", "voronoi1024_pd5_vd3"):
        img = voronoi_image(1024, 1024, 200, s + 3)
        f = spatial_rgb_features(img, 32.0, 0.08)
        v = img if name.endswith("vd3") else np.concatenate(
            [img, np.ones(img.shape[:2] + (1,), np.float32)], axis=-1)
    elif name in ("gauss512_pd16_vd8", "gauss256_pd16_vd8"):
        n = 512 if name.startswith("gauss512") else 256
        rng = np.random.default_rng(s + 4)
        f = (rng.standard_normal((n, n, 16)) * 2.0).astype(np.float32)
        v = rng.uniform(-1.0, 1.0, (n, n, 8)).astype(np.float32)
    elif name == "collapse512_pd2_vd8":
        rng = np.random.default_rng(s + 5)
        f = np.empty((512, 512, 2), np.float32)
        f[..., 0], f[..., 1] = 0.3, 0.7
        v = rng.uniform(-1.0, 1.0, (512, 512, 8)).astype(np.float32)
    elif name == "crf512_pd5_vd3":
        k = s + 6 + index
        img = blob_image(512, 512, 64, k) if index % 2 == 0 else voronoi_image(512, 512, 200, k)
        f = spatial_rgb_features(img, 20.0, 0.1)
        v = _softmax3(np.random.default_rng(k + 7), 512, 512)
    else:
        raise KeyError(f"unknown workload {name!r}; known: {sorted(WORKLOADS)}")
    g = _grad(np.random.default_rng(s + 99 + 7 * index), v.shape)
    return {"features": np.ascontiguousarray(f, np.float32),
            "values": np.ascontiguousarray(v, np.float32),
            "grad": g}


WORKLOADS = {
    "blobs64_pd5_vd3": (64, 64, 5, 3),
    "blobs256_pd5_vd3": (256, 256, 5, 3),
    "voronoi1024_pd5_vd4": (1024, 1024, 5, 4),
    "voronoi1024_pd5_vd3": (1024, 1024, 5, 3),
    "gauss512_pd16_vd8": (512, 512, 16, 8),
    "gauss256_pd16_vd8": (256, 256, 16, 8),
    "collapse512_pd2_vd8": (512, 512, 2, 8),
    "crf512_pd5_vd3": (512, 512, 5, 3),
}
