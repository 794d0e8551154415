"""Invariants of the lattice the sm_100a build leaves in its buffers.

The parity tests compare what the filter returns; these read the lattice and
scratch buffers of one forward call back to the host and check the structure
every later kernel relies on, for every feature dimension:
  * every vertex key record has its padding halfwords zero and word 0 equal to
    the hash of its coordinates (lookups compare whole records, so a record
    that decodes to the right coordinates but differs anywhere else is not
    found; neighbour hashes are derived incrementally from that hash);
  * every (pixel, simplex corner) slot resolves to the vertex whose key the
    oracle's embedding gives (permutohedral.cu:238-244), with the same weight;
  * each tile's slots, counting-sorted by local vertex id, cover the tile's
    active slots exactly once, in runs of one id each with the run starts
    flagged, and the first id of every K positions is recorded;
  * the blur neighbour table holds, per axis and direction, the vertex whose
    key is the step of permutohedral.cu:368-375 away, or -1 where there is none.
The buffer layout is restated here and checked against the library's own
workspace sizes, so that a change of layout fails loudly instead of being
misread.
"""
import os

import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN, golden_files

pytestmark = pytest.mark.gpu


def _align(x):
    return (x + 255) & ~255


def _pad_ch(c):
    return c if c <= 2 else ((c + 3) // 4) * 4


def _layout(h, w, pd, vd):
    K = pd + 1
    P = 256 if pd <= 6 else (128 if pd <= 10 else 64)
    TH = P // 32
    tx = (w + 31) // 32
    T = tx * ((h + TH - 1) // TH)
    CW = (4 + 2 * pd + 15) // 16
    CPf, CPb = _pad_ch(vd + 1), _pad_ch(vd)
    S = T * K * P
    lg = 6
    while (1 << lg) < 2 * S:
        lg += 1
    lat, o = {}, _align(256)
    for name, sz in [("tile_off", T * 4), ("tile_cnt", T * 4), ("slot_lid", S * 2), ("slot_w", S * 4),
                     ("slot_order", S * 2), ("slot_wsort", S * 4), ("first_lid", T * P * 2), ("staged_vid", S * 4),
                     ("nbr", S * K * 8), ("vb0", S * CPb * 4)]:
        lat[name] = o
        o = _align(o + sz)
    lat_bytes, scr, o = o, {}, 0
    # scratch: the value rows and the blur's bookkeeping (front part), then the build part
    for name, sz in [("v1", S * CPf * 4), ("bstate", 2 * S), ("v0", S * CPf * 4),
                     ("skeys", S * CW * 16), ("table", (1 << lg) * 4), ("filter", 1 << lg), ("owner", S * 4),
                     ("vid_of", S * 4), ("vkeys", S * CW * 16)]:
        scr[name] = o
        o = _align(o + sz)
    return lat, scr, dict(K=K, P=P, TH=TH, tx=tx, T=T, CW=CW, S=S, lat_bytes=lat_bytes, scr_bytes=o)


def _view(buf, off, n, dt):
    return buf[off:off + n * np.dtype(dt).itemsize].view(dt)


_COORD_MUL = [0x2AE75E2F, 0x9C2B9D9F, 0x4F876AA3, 0x02FF349D, 0xBAEC4EF7, 0xE06C85AF, 0x21F64545, 0xE7158A81,
              0x819ED6B7, 0x3C95AD21, 0x8BE9794D, 0x3C7BA9E3, 0x022DD18D, 0x4D317C69, 0x7965C0FF, 0x8ECA7365]


def _key_hash(words, pd):
    """Hash of key records [n][NW] as the device computes it: the sum of the
    sign-extended int16 coordinates times per-coordinate odd multipliers
    (mod 2^32), then an avalanche (fmix32)."""
    m32 = np.uint64(0xFFFFFFFF)
    coords, _ = _decode(words, pd)
    lin = np.zeros(words.shape[0], np.uint64)
    for i in range(pd):
        c = coords[:, i].astype(np.int64) & 0xFFFFFFFF
        lin = (lin + c.astype(np.uint64) * np.uint64(_COORD_MUL[i])) & m32
    h = lin ^ np.uint64(0x9E3779B9)
    h ^= h >> np.uint64(16)
    h = (h * np.uint64(0x85EBCA6B)) & m32
    h ^= h >> np.uint64(13)
    h = (h * np.uint64(0xC2B2AE35)) & m32
    h ^= h >> np.uint64(16)
    return h.astype(np.uint32)


def _decode(words, pd):
    """int16 coordinates [n][pd] and the OR of the padding halfwords [n]."""
    half = np.stack([(words[:, 1:] >> np.uint32(16 * s)) & np.uint32(0xFFFF) for s in (0, 1)], axis=2)
    half = half.reshape(words.shape[0], -1)
    return half[:, :pd].astype(np.uint16).view(np.int16), np.bitwise_or.reduce(half[:, pd:], axis=1)


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from plattice_pytorch_b200 import _lib
    _lib.lib()
    return torch.device("cuda:0")


CASES = [f for f in golden_files() if f.startswith("ref_randn24x20_")] + ["ref_ragged13x29_pd5_vd3.npz"]


@pytest.mark.parametrize("fn", CASES)
def test_lattice_invariants(fn, dev):
    _check_invariants(fn, dev)


@pytest.mark.parametrize("fn", ["ref_randn24x20_pd2_vd3.npz", "ref_randn24x20_pd5_vd6.npz",
                                "ref_randn24x20_pd16_vd1.npz", "ref_ragged13x29_pd5_vd3.npz"])
def test_lattice_invariants_with_miss_filter(fn, dev):
    """The neighbour lookups through the miss filter, which by default only
    large tables use, forced on for small ones: the same exact neighbours."""
    from plattice_pytorch_b200 import _lib
    L = _lib.lib()
    try:
        L.plattice_debug_set_miss_filter_log2(6)
        _check_invariants(fn, dev)
    finally:
        L.plattice_debug_set_miss_filter_log2(0)


def _check_invariants(fn, dev):
    from plattice_pytorch_b200 import PLOO, _lib
    d = np.load(os.path.join(GOLDEN, fn))
    f, v = d["features"], d["values"]
    h, w, pd = f.shape
    vd = v.shape[2]
    lat_off, scr_off, g = _layout(h, w, pd, vd)
    assert (g["lat_bytes"], g["scr_bytes"]) == tuple(_lib.workspace_sizes(h, w, pd, vd))
    K, P, TH, tx, T, CW, S = (g[k] for k in ("K", "P", "TH", "tx", "T", "CW", "S"))

    _, _, lat = PLOO.lattice_forward(torch.from_numpy(f).to(dev), torch.from_numpy(v).to(dev), keep_scratch=True)
    torch.cuda.synchronize()
    lb, sb = lat.buf.cpu().numpy(), lat.scratch.cpu().numpy()
    hdr = lb[:256].view(np.int32)
    assert hdr[0] == 0
    M, U = int(hdr[1]), int(hdr[2])

    # key records: padding zero, hash consistent, all distinct
    for name, n in (("vkeys", M), ("skeys", U)):
        words = _view(sb, scr_off[name], n * CW * 4, np.uint32).reshape(n, CW * 4)
        coords, padding = _decode(words, pd)
        assert not padding.any(), (name, int(np.count_nonzero(padding)))
        assert np.array_equal(words[:, 0], _key_hash(words, pd)), name
    vk, _ = _decode(_view(sb, scr_off["vkeys"], M * CW * 4, np.uint32).reshape(M, CW * 4), pd)
    assert len({r.tobytes() for r in vk}) == M
    vid_of_key = {r.tobytes(): i for i, r in enumerate(vk)}

    # slots against the oracle's embedding
    tile_off = _view(lb, lat_off["tile_off"], T, np.int32)
    tile_cnt = _view(lb, lat_off["tile_cnt"], T, np.int32)
    slot_lid = _view(lb, lat_off["slot_lid"], S, np.uint16).reshape(T, K, P)
    slot_w = _view(lb, lat_off["slot_w"], S, np.float32).reshape(T, K, P)
    order = _view(lb, lat_off["slot_order"], S, np.uint16).reshape(T, K * P)
    wsort = _view(lb, lat_off["slot_wsort"], S, np.float32).reshape(T, K * P)
    first_lid = _view(lb, lat_off["first_lid"], T * P, np.uint16).reshape(T, P)
    staged_vid = _view(lb, lat_off["staged_vid"], S, np.int32)
    okeys, ow = oracle.embed(f)
    okeys = okeys.reshape(h * w, K, pd)
    ow = ow.reshape(h * w, K)
    assert int(tile_cnt.sum()) == U
    for tile in range(T):
        ts = np.arange(P)
        xs = (tile % tx) * 32 + ts % 32
        ys = (tile // tx) * TH + ts // 32
        act = ts[(xs < w) & (ys < h)]
        base, cnt = int(tile_off[tile]), int(tile_cnt[tile])
        for t in act:
            p = int(ys[t]) * w + int(xs[t])
            for c in range(K):
                lid = int(slot_lid[tile, c, t])
                assert lid < cnt
                assert staged_vid[base + lid] == vid_of_key[okeys[p, c].tobytes()], (tile, t, c)
                assert slot_w[tile, c, t].view(np.uint32) == ow[p, c].view(np.uint32), (tile, t, c)
        # sorted order: runs of equal local id in id order, each entry (pixel, run start)
        total = len(act) * K
        seen = set()
        u = -1
        for pos in range(total):
            e = int(order[tile, pos])
            t, start = e >> 1, e & 1
            assert start == (1 if pos == 0 else start)
            u += start
            cs = [c for c in range(K) if slot_lid[tile, c, t] == u]
            assert len(cs) == 1 and (t, cs[0]) not in seen, (tile, pos)
            assert wsort[tile, pos].view(np.uint32) == slot_w[tile, cs[0], t].view(np.uint32)
            seen.add((t, cs[0]))
            if pos % K == 0:
                assert first_lid[tile, pos // K] == u, (tile, pos)
        assert len(seen) == total and u + 1 == cnt

    # blur neighbours
    nbr = _view(lb, lat_off["nbr"], M * K * 2, np.int32).reshape(K, M, 2)
    for c in range(K):
        step = np.ones(pd, np.int32)
        if c < pd:
            step[c] -= K
        for col, sgn in ((0, 1), (1, -1)):
            nk = (vk.astype(np.int32) + sgn * step).astype(np.int16)
            expect = np.array([vid_of_key.get(r.tobytes(), -1) for r in nk], np.int32)
            assert np.array_equal(nbr[c, :, col], expect), (c, sgn, int(np.count_nonzero(nbr[c, :, col] != expect)))


def _neighbour_keys(f, v, dev):
    """Vertex keys [M, pd] sorted, and for each of them and each (axis, direction)
    the neighbour's key, or a row of the int16 minimum where there is none."""
    from plattice_pytorch_b200 import PLOO
    h, w, pd = f.shape
    lat_off, scr_off, g = _layout(h, w, pd, v.shape[2])
    K, CW = g["K"], g["CW"]
    _, _, lat = PLOO.lattice_forward(torch.from_numpy(f).to(dev), torch.from_numpy(v).to(dev), keep_scratch=True)
    torch.cuda.synchronize()
    assert PLOO.lattice_info(lat)["status"] == 0
    lb, sb = lat.buf.cpu().numpy(), lat.scratch.cpu().numpy()
    M = int(lb[:256].view(np.int32)[1])
    vk, _ = _decode(_view(sb, scr_off["vkeys"], M * CW * 4, np.uint32).reshape(M, CW * 4), pd)
    nbr = _view(lb, lat_off["nbr"], M * K * 2, np.int32).reshape(K, M, 2)
    none = np.full((1, pd), -32768, np.int16)
    table = np.concatenate([vk, none])                    # index -1 -> the sentinel row
    nk = table[np.where(nbr < 0, M, nbr)]                 # [K, M, 2, pd]
    order = np.lexsort(vk.T[::-1])
    return vk[order], nk[:, order]


def test_sparse_neighbour_path_matches_dense(dev):
    """A lattice large enough for one vertex per thread, with the miss filter
    forced on, takes the sparse neighbour path (first sweep, per-warp queue);
    with the filter off the dense path.  Both give the same neighbours."""
    from plattice_pytorch_b200 import _lib
    rng = np.random.default_rng(7)
    f = (rng.normal(size=(192, 192, 16)) * 2.0).astype(np.float32)   # about 627 k distinct vertices
    v = rng.uniform(-1.0, 1.0, size=(192, 192, 1)).astype(np.float32)
    L = _lib.lib()
    try:
        L.plattice_debug_set_miss_filter_log2(6)
        keys_s, nk_s = _neighbour_keys(f, v, dev)
        L.plattice_debug_set_miss_filter_log2(30)
        keys_d, nk_d = _neighbour_keys(f, v, dev)
    finally:
        L.plattice_debug_set_miss_filter_log2(0)
    assert keys_s.shape[0] > 148 * 8 * 256   # more vertices than the neighbour grid's threads
    assert np.array_equal(keys_s, keys_d)
    assert np.array_equal(nk_s, nk_d)
    assert (nk_s[..., 0] != -32768).mean() > 0.01   # some neighbours exist
