"""numpy restatement of the per-sample static geometry (test oracle only).

Every function cites the reference code it restates (paths relative to the
reference project; ``BK/`` = ``baseline_repo/3dgen-main/``).  Integer outputs
are bit-exact with the reference; RoPE tables follow its fp64->fp32 recipe.
"""
from __future__ import annotations

import numpy as np

ORDERS = ("h", "ht1", "h1", "ht")  # weights/config.json model_config.orders


def lex_perm(vox: np.ndarray):
    """SparseDownsample(patch=1) ordering of one sample.

    Restates ``lib/fast_flow.py:667-694`` (key = x<<20 | y<<10 | z, argsort,
    inverse) which equals ``BK/base_models/sparse.py:998-1036`` for unique
    coordinates below 1024.  Returns (perm, up_widx, h_coords[N,4] int32 with
    batch column 0).
    """
    v = np.asarray(vox).astype(np.int64)
    key = (v[:, 0] << 20) | (v[:, 1] << 10) | v[:, 2]
    perm = np.argsort(key, kind="stable").astype(np.int64)
    up = np.empty_like(perm)
    up[perm] = np.arange(len(perm), dtype=np.int64)
    hc = np.zeros((len(v), 4), dtype=np.int32)
    hc[:, 1:] = v[perm]
    return perm, up, hc


def _split_by_3(a: np.ndarray) -> np.ndarray:
    """Bit interleave helper of ``lib/fast_kernels.py:201-208`` (21 bits)."""
    w = a.astype(np.uint64) & np.uint64(0x1FFFFF)
    w = (w | (w << np.uint64(32))) & np.uint64(0x001F00000000FFFF)
    w = (w | (w << np.uint64(16))) & np.uint64(0x001F0000FF0000FF)
    w = (w | (w << np.uint64(8))) & np.uint64(0x010F00F00F00F00F)
    w = (w | (w << np.uint64(4))) & np.uint64(0x10C30C30C30C30C3)
    w = (w | (w << np.uint64(2))) & np.uint64(0x1249249249249249)
    return w


def hilbert3(x: np.ndarray, y: np.ndarray, z: np.ndarray) -> np.ndarray:
    """16-level 3D Hilbert distance, ``BK/base_models/order.py:6-53``.

    The loop runs i = 15..1 regardless of the coordinate range (the
    orientation of the low bits depends on it); the output interleaves
    x,y,z bits as (x<<2 | y<<1 | z) per level.
    """
    x = x.astype(np.int64).copy()
    y = y.astype(np.int64).copy()
    z = z.astype(np.int64).copy()
    for i in range(15, 0, -1):
        q = np.int64(1 << i)
        p = np.int64((1 << i) - 1)
        x = np.where((x & q) > 0, x ^ p, x)
        cond = (y & q) > 0
        t = (x ^ y) & p
        x = x ^ np.where(cond, p, t)
        y = y ^ np.where(cond, 0, t)
        cond = (z & q) > 0
        t = (x ^ z) & p
        x = x ^ np.where(cond, p, t)
        z = z ^ np.where(cond, 0, t)
    y ^= x
    z ^= y
    t = np.zeros_like(z)
    for i in range(15, 0, -1):
        q = np.int64(1 << i)
        t = t ^ np.where((z & q) > 0, q - 1, 0)
    x ^= t
    y ^= t
    z ^= t
    ret = (_split_by_3(x) << np.uint64(2)) | (_split_by_3(y) << np.uint64(1)) | _split_by_3(z)
    return ret.astype(np.int64)


def encode_orders4(h_coords: np.ndarray) -> np.ndarray:
    """Codes of the four window orders (h, ht1, h1, ht) -> [4, N] int64.

    Follows the fused encoder ``lib/fast_kernels.py:1126-1154``: ``*1``
    orders add 1 to x, y, z only; ``t`` orders swap x and y; the batch index
    is OR-ed in at bit 48.
    """
    hc = np.asarray(h_coords).astype(np.int64)
    b = hc[:, 0] << 48
    x, y, z = hc[:, 1], hc[:, 2], hc[:, 3]
    return np.stack([
        hilbert3(x, y, z) | b,
        hilbert3(y + 1, x + 1, z + 1) | b,
        hilbert3(x + 1, y + 1, z + 1) | b,
        hilbert3(y, x, z) | b,
    ])


def order_caches(codes4: np.ndarray):
    """fwd = argsort(code), bwd = inverse (``lib/fast_kernels.py:1816-1822``).

    Codes are unique per voxel (the Hilbert map is a bijection), so every
    correct sort yields this permutation.
    """
    out = []
    n = codes4.shape[1]
    for c in codes4:
        fwd = np.argsort(c, kind="stable").astype(np.int64)
        bwd = np.empty_like(fwd)
        bwd[fwd] = np.arange(n, dtype=np.int64)
        out.append((fwd, bwd))
    return out


def window_cu_seqlens(n: int, patch_size: int = 4096) -> np.ndarray:
    """Window partition of one sample, ``lib/fast_kernels.py:1764-1790``."""
    lens = []
    if n > 0:
        full = (n - 1) // patch_size
        lens = [patch_size] * full + [n - full * patch_size]
    return np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)


def conv_offset(d: int):
    """Offset of tap d, ``BK/ops/libsparse/conv.cu:64-72`` (d = (dx+1)*9+(dy+1)*3+(dz+1))."""
    return d // 9 - 1, (d // 3) % 3 - 1, d % 3 - 1


def conv_indices(h_coords: np.ndarray) -> np.ndarray:
    """27-neighbour index table [N,27] int32 with -1 for absent neighbours.

    Restates ``BK/ops/libsparse/conv.cu:74-163`` / ``lib/fast_kernels.py:1649-1701``:
    key = b<<36 | x<<24 | y<<12 | z; each neighbour with non-negative
    coordinates is looked up among the sorted keys; the result indexes rows of
    ``h_coords``.
    """
    hc = np.asarray(h_coords).astype(np.int64)
    b, x, y, z = hc[:, 0], hc[:, 1], hc[:, 2], hc[:, 3]
    keys = (b << 36) | (x << 24) | (y << 12) | z
    order = np.argsort(keys, kind="stable")
    sk = keys[order]
    n = len(hc)
    out = np.full((n, 27), -1, dtype=np.int32)
    for d in range(27):
        dx, dy, dz = conv_offset(d)
        xx, yy, zz = x + dx, y + dy, z + dz
        valid = (xx >= 0) & (yy >= 0) & (zz >= 0)
        q = (b << 36) | (np.maximum(xx, 0) << 24) | (np.maximum(yy, 0) << 12) | np.maximum(zz, 0)
        pos = np.searchsorted(sk, q)
        posc = np.minimum(pos, n - 1)
        found = valid & (pos < n) & (sk[posc] == q) if n else valid
        out[found, d] = order[posc[found]].astype(np.int32)
    return out


def rope3d_table(res: int, head_dim: int, base: float = 128.0):
    """[res, M] cos/sin, M = head_dim // 6 (``lib/fast_kernels.py:977-993``).

    pos = (c + 0.5) / res * 2 - 1, inv_freq = base^(-i/M), fp64 then fp32.
    """
    m = head_dim // 6
    c = (np.arange(res, dtype=np.float64) + 0.5) / float(res) * 2.0 - 1.0
    inv = float(base) ** (-np.arange(m, dtype=np.float64) / float(m))
    f = c[:, None] * inv[None, :]
    return np.cos(f).astype(np.float32), np.sin(f).astype(np.float32)


def rope2d_table(cond_size: int, head_dim: int, base: float = 64.0):
    """[cond_size^2, 2, M] cos/sin, M = head_dim // 4 (``lib/fast_kernels.py:1011-1035``).

    Token t = i*cond_size + j has positions (i, j) (meshgrid 'ij',
    ``BK/models/generators/lat_dit.py:546-555``).
    """
    m = head_dim // 4
    ii, jj = np.meshgrid(np.arange(cond_size), np.arange(cond_size), indexing="ij")
    pos = np.stack([ii.reshape(-1), jj.reshape(-1)], -1).astype(np.float64)
    pos = (pos + 0.5) / float(cond_size) * 2.0 - 1.0
    inv = float(base) ** (-np.arange(m, dtype=np.float64) / float(m))
    f = pos[:, :, None] * inv[None, None, :]
    return np.cos(f).astype(np.float32), np.sin(f).astype(np.float32)


def sample_geometry(vox: np.ndarray, patch_size: int = 4096):
    """All static geometry of one sample, mirroring ``_prepare_sample_geometry``
    (``lib/fast_flow.py:657-783``)."""
    perm, up, hc = lex_perm(vox)
    codes = encode_orders4(hc)
    caches = order_caches(codes)
    return {
        "perm": perm, "up_widx": up, "h_coords": hc, "codes4": codes,
        "order_caches": caches, "cu_seqlens": window_cu_seqlens(len(hc), patch_size),
        "conv_indices": conv_indices(hc),
    }
