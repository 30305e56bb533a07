"""Oracle: tile map, spatial-hash binning and the slot->gaussian inverse table (numpy).

Restates ``tools/m4_train_binned.py:60-127`` (TileMap, assign_bins) and
``tools/m9_scatter_oracle.py:20-42`` (build_inv, gather_reduce) in numpy with the exact fp32
arithmetic of the reference, so that the binning tables compare bit for bit.

Canonical order: the reference sorts the packed key ``tile*2048 + clamp(long(dist2), 0, 2047)``
with ``torch.argsort`` (``tools/m4_train_binned.py:115``), which is not stable on every size.
The canonical order used for bit-exact comparison is the *stable* sort of that key, i.e. ties on
the quantised distance are broken by the reference's input order: stencil offset index
``j = (dy+R)*(2R+1) + (dx+R)`` ascending (the dy/dx loop at ``:92-98``), then gaussian id
ascending.  ``stable=False`` reproduces numpy's default (quicksort) for comparison only.

Float->int64 conversion: on this torch build ``Tensor.long()`` maps non-finite values and
values outside [-2^63, 2^63) to INT64_MIN (probed); the cell index and the quantised distance
both then clamp to 0.  ``_to_long`` restates that.
"""
from types import SimpleNamespace

import numpy as np

_I64_MIN = np.iinfo(np.int64).min
_TWO63 = np.float32(2.0 ** 63)


def tile_map(H, W):
    """TileMap (tools/m4_train_binned.py:60-72): 16x16 tiles, tile-local Phi at pixel centres,
    tile origins, and the tile-pixel -> row-major image index ``gidx``."""
    assert H % 16 == 0 and W % 16 == 0
    nty, ntx = H // 16, W // 16
    T = nty * ntx
    p = np.arange(256)
    lx = (p % 16).astype(np.float32) + np.float32(0.5)
    ly = (p // 16).astype(np.float32) + np.float32(0.5)
    # forward.phi (spike/forward.py:42-44): [px^2, py^2, px*py, px, py, 1]
    Phi = np.stack([lx * lx, ly * ly, lx * ly, lx, ly, np.ones_like(lx)], -1).astype(np.float32)
    t = np.arange(T)
    ty, tx = t // ntx, t % ntx
    origins = np.stack([(tx * 16).astype(np.float32), (ty * 16).astype(np.float32)], 1)
    gr = ty[:, None] * 16 + (p // 16)[None, :]
    gc = tx[:, None] * 16 + (p % 16)[None, :]
    gidx = (gr * W + gc).reshape(-1).astype(np.int64)
    return SimpleNamespace(H=H, W=W, nty=nty, ntx=ntx, T=T, Phi=Phi, origins=origins, gidx=gidx)


def _to_long(x):
    """torch ``Tensor.long()`` on float32: truncation, INT64_MIN when not in [-2^63, 2^63)."""
    x = np.asarray(x, np.float32)
    ok = (x >= -_TWO63) & (x < _TWO63)
    out = np.full(x.shape, _I64_MIN, np.int64)
    out[ok] = x[ok].astype(np.int64)
    return out


def cells(mu2d, ntx, nty):
    """Home cell of each gaussian (tools/m4_train_binned.py:85-86): floor(mu/16), clamped into
    the grid, so off-screen gaussians land in border cells."""
    mu2d = np.asarray(mu2d, np.float32)
    gx = np.clip(_to_long(np.floor(mu2d[:, 0] / np.float32(16))), 0, ntx - 1)
    gy = np.clip(_to_long(np.floor(mu2d[:, 1] / np.float32(16))), 0, nty - 1)
    return gx, gy


def quantised_dist2(mu2d, tiles, ntx):
    """dist2 to the tile centre in fp32 and its clamp(long(.), 0, 2047) quantisation
    (tools/m4_train_binned.py:110-114)."""
    tx_f = (tiles % ntx).astype(np.float32)
    ty_f = (tiles // ntx).astype(np.float32)
    dx = mu2d[:, 0] - (tx_f + np.float32(0.5)) * np.float32(16.0)
    dy = mu2d[:, 1] - (ty_f + np.float32(0.5)) * np.float32(16.0)
    d2 = dx * dx + dy * dy
    return d2, np.clip(_to_long(d2), 0, 2047)


def candidate_pairs(mu2d, keep, tm, R):
    """The (tile, gaussian, stencil j) pairs in the reference's input order
    (tools/m4_train_binned.py:90-106): dy outer, dx inner, gaussians ascending."""
    mu2d = np.asarray(mu2d, np.float32)
    keep = np.asarray(keep, bool)
    G = mu2d.shape[0]
    gx, gy = cells(mu2d, tm.ntx, tm.nty)
    g_all = np.arange(G)
    tiles_l, gs_l, js_l = [], [], []
    j = 0
    for dy in range(-R, R + 1):
        for dx in range(-R, R + 1):
            txn, tyn = gx + dx, gy + dy
            ok = keep & (txn >= 0) & (txn < tm.ntx) & (tyn >= 0) & (tyn < tm.nty)
            tiles_l.append((tyn * tm.ntx + txn)[ok])
            gs_l.append(g_all[ok])
            js_l.append(np.full(int(ok.sum()), j, np.int64))
            j += 1
    return np.concatenate(tiles_l), np.concatenate(gs_l), np.concatenate(js_l)


def assign_bins(mu2d, keep, tm, R, K, stable=True):
    """assign_bins (tools/m4_train_binned.py:75-127).

    Returns a namespace with ``idx[T,K]`` int64 (0 in invalid slots, like the reference),
    ``valid[T,K]`` bool, ``count[T] = min(cand, K)``, ``cand[T]`` (candidates per tile; overflow
    is ``max(0, cand - K)``), ``slot_j[T,K]`` (stencil index of each kept slot, -1 if invalid)
    and ``q[T,K]`` (its quantised distance)."""
    mu2d = np.asarray(mu2d, np.float32)
    T = tm.T
    idx = np.zeros((T, K), np.int64)
    valid = np.zeros((T, K), bool)
    slot_j = np.full((T, K), -1, np.int64)
    slot_q = np.full((T, K), -1, np.int64)
    tiles, gs, js = candidate_pairs(mu2d, keep, tm, R)
    cand = np.bincount(tiles, minlength=T).astype(np.int64)
    if tiles.size:
        _, q = quantised_dist2(mu2d[gs], tiles, tm.ntx)
        key = tiles.astype(np.int64) * 2048 + q
        order = np.argsort(key, kind="stable" if stable else "quicksort")
        tiles, gs, js, q = tiles[order], gs[order], js[order], q[order]
        start = np.searchsorted(tiles, np.arange(T + 1))
        pos = np.arange(tiles.size) - start[tiles]
        m = pos < K
        flat = tiles[m] * K + pos[m]
        idx.reshape(-1)[flat] = gs[m]
        valid.reshape(-1)[flat] = True
        slot_j.reshape(-1)[flat] = js[m]
        slot_q.reshape(-1)[flat] = q[m]
    count = valid.sum(1).astype(np.int64)
    return SimpleNamespace(idx=idx, valid=valid, count=count, cand=cand, slot_j=slot_j, q=slot_q)


def build_inv(idx, valid, G, Smax):
    """build_inv (tools/m9_scatter_oracle.py:20-35): per gaussian, its valid slot positions in
    ascending flat order, padded with the sentinel T*K."""
    TK = idx.size
    flat_idx = idx.reshape(-1)
    slots = np.nonzero(valid.reshape(-1))[0]
    g_of = flat_idx[slots]
    order = np.argsort(g_of, kind="stable")
    g_s, slot_s = g_of[order], slots[order]
    counts = np.bincount(g_of, minlength=G)
    assert counts.size == 0 or int(counts.max()) <= Smax
    csum = np.cumsum(counts) - counts
    within = np.arange(g_s.size) - csum[g_s]
    inv = np.full((G, Smax), TK, np.int64)
    inv[g_s, within] = slot_s
    return inv


def stencil_inv(bins, G, R):
    """The inverse table indexed by stencil offset: ``inv[g, j]`` = flat slot position
    ``t*K + k`` of gaussian g in the tile at its stencil offset j, or -1.  Holds the same
    per-gaussian slot SET as ``build_inv`` (the layout the device reduction consumes)."""
    S = (2 * R + 1) ** 2
    T, K = bins.idx.shape
    inv = np.full((G, S), -1, np.int64)
    flat = np.nonzero(bins.valid.reshape(-1))[0]
    inv[bins.idx.reshape(-1)[flat], bins.slot_j.reshape(-1)[flat]] = flat
    return inv


def gather_reduce(grad_slots, inv_pad):
    """gather_reduce (tools/m9_scatter_oracle.py:38-42) over a sentinel-padded inverse table."""
    T, K, C = grad_slots.shape
    pad = np.concatenate([grad_slots.reshape(T * K, C), np.zeros((1, C), grad_slots.dtype)], 0)
    return pad[inv_pad.reshape(-1)].reshape(inv_pad.shape[0], inv_pad.shape[1], C).sum(1)


def table_digest(bins):
    """sha256 over (idx with -1 in invalid slots as int32, count, cand) for compact fixtures."""
    import hashlib
    idx = np.where(bins.valid, bins.idx, -1).astype(np.int32)
    h = hashlib.sha256()
    h.update(np.ascontiguousarray(idx).tobytes())
    h.update(np.ascontiguousarray(bins.count.astype(np.int32)).tobytes())
    h.update(np.ascontiguousarray(bins.cand.astype(np.int32)).tobytes())
    return h.hexdigest()
