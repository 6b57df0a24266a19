"""Host wrappers of the sm_100a kernels, under the reference's ``lib/fast_kernels.py`` names.

Each function allocates its outputs with torch (device memory is torch's
caching allocator), launches on the current CUDA stream through the C ABI
and raises on any error.  There is no CPU or Triton path.

Reference names kept: ``precompute_rope_3d_table``, ``precompute_rope_2d_cond``,
``build_order_caches_fast``, ``build_conv_indices_fast``, ``fast_sparse_conv3d``,
``fast_modulate``, ``fast_gate_add_and_modulate``, ``fast_gate_add``,
``fused_qknorm_rope3d_gather``, ``fused_qknorm_rope2d_cond_inplace``,
``fast_swiglu_from_packed``, ``fast_out_modulate_unpatchify``,
``flash_varlen_qkvpacked_already_sorted``, ``flash_cross_attn``,
``flash_cond_self_attn``.
"""
from __future__ import annotations

import ctypes
import math
from typing import List, Optional, Sequence, Tuple

import torch

from ._lib import check, lib, ptr, stream_of

BF16 = torch.bfloat16


def _s(t: torch.Tensor) -> int:
    return stream_of(t)


def _f32(v: torch.Tensor) -> torch.Tensor:
    return v.reshape(-1).to(torch.float32).contiguous()


# ----------------------------------------------------------------------------- geometry

def lex_perm(vox: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(perm, up_widx, h_coords) of one sample, ``lib/fast_flow.py:667-694``."""
    if vox.dim() != 2 or vox.shape[1] != 3:
        raise ValueError(f"voxel coordinates must be [N, 3] (x, y, z), got {tuple(vox.shape)}")
    vox = vox.to(torch.int32).contiguous()
    n = vox.shape[0]
    dev = vox.device
    perm = torch.empty(n, dtype=torch.int64, device=dev)
    up = torch.empty(n, dtype=torch.int64, device=dev)
    hc = torch.empty(n, 4, dtype=torch.int32, device=dev)
    ws = torch.empty(int(lib().vdit_geometry_workspace_bytes(n)), dtype=torch.uint8, device=dev)
    check(lib().vdit_lex_perm(ptr(vox), n, ptr(perm), ptr(up), ptr(hc), ptr(ws), ws.numel(), _s(vox)), "lex_perm")
    return perm, up, hc


def hilbert4_orders(h_coords: torch.Tensor, coord_bound: int, return_codes: bool = False):
    """Codes and (fwd, bwd) permutations of the orders (h, ht1, h1, ht)."""
    h_coords = h_coords.to(torch.int32).contiguous()
    n = h_coords.shape[0]
    dev = h_coords.device
    fwd = torch.empty(4, n, dtype=torch.int64, device=dev)
    bwd = torch.empty(4, n, dtype=torch.int64, device=dev)
    codes = torch.empty(4, n, dtype=torch.int64, device=dev) if return_codes else None
    ws = torch.empty(int(lib().vdit_geometry_workspace_bytes(n)), dtype=torch.uint8, device=dev)
    check(lib().vdit_hilbert4_orders(ptr(h_coords), n, int(coord_bound), ptr(codes), ptr(fwd), ptr(bwd), ptr(ws),
                                     ws.numel(), _s(h_coords)), "hilbert4_orders")
    return (codes, fwd, bwd) if return_codes else (fwd, bwd)


def window_seqlens(sizes: Sequence[int], patch_size: int) -> Tuple[List[int], int]:
    """Host-side window partition, ``lib/fast_kernels.py:1764-1790``."""
    lens: List[int] = []
    for s in sizes:
        s = int(s)
        if s > 0:
            full = (s - 1) // patch_size
            lens += [patch_size] * full + [s - full * patch_size]
    cu = [0]
    for v in lens:
        cu.append(cu[-1] + v)
    return cu, (max(lens) if lens else 0)


def build_order_caches_fast(h_coords: torch.Tensor, sizes: List[int], orders: Sequence[str], order_kwargs: dict,
                            seqlen_cache: Optional[dict] = None, arange_n: Optional[torch.Tensor] = None,
                            use_triton: bool = True, coord_bound: Optional[int] = None):
    """Four Hilbert window orders of one sample -> [(fwd, bwd, cu_seqlens, max_len)] * 4
    (``lib/fast_kernels.py:1739-1836``; ``use_triton`` is accepted and ignored).
    ``cu_seqlens`` is returned as a device int32 tensor carrying a host copy in
    ``.host`` (the attention launch needs the window sizes on the host)."""
    if tuple(orders) != ("h", "ht1", "h1", "ht"):
        raise NotImplementedError(f"orders {tuple(orders)}: only ('h', 'ht1', 'h1', 'ht') is built")
    if len(sizes) != 1:
        raise NotImplementedError("one sample per geometry")
    patch = int(order_kwargs.get("patch_size", 4096))
    cu, max_len = window_seqlens(sizes, patch)
    if coord_bound is None:
        coord_bound = int(h_coords[:, 1:].max().item()) + 1 if h_coords.numel() else 1
    fwd, bwd = hilbert4_orders(h_coords, coord_bound)
    cu_t = torch.tensor(cu, dtype=torch.int32, device=h_coords.device)
    cu_t.host = cu
    return [(fwd[i], bwd[i], cu_t, max_len) for i in range(4)]


def build_conv_indices_fast(coords: torch.Tensor, already_sorted: bool = False) -> List[torch.Tensor]:
    """27-neighbour indices [N,27] int32 (-1 absent), ``lib/fast_kernels.py:1649-1701``."""
    coords = coords.to(torch.int32).contiguous()
    n = coords.shape[0]
    if already_sorted:
        out = torch.empty(n, 27, dtype=torch.int32, device=coords.device)
        check(lib().vdit_conv_indices(ptr(coords), n, ptr(out), _s(coords)), "conv_indices")
        return [out]
    if n and int(coords[:, 0].max().item()) != 0:
        raise NotImplementedError("unsorted coordinates of several samples")
    perm, up, hc = lex_perm(coords[:, 1:].contiguous())
    sorted_idx = build_conv_indices_fast(hc, already_sorted=True)[0]
    # rows back to input order, neighbour ids back to input ids
    idx = sorted_idx[up]
    out = torch.where(idx >= 0, perm[idx.clamp(min=0).long()].to(torch.int32), idx)
    return [out.contiguous()]


def precompute_rope_3d_table(res: int = 64, base: float = 128.0, head_dim: int = 96,
                             device: Optional[torch.device] = None):
    """[res, head_dim//6] cos/sin (fp64 -> fp32), ``lib/fast_kernels.py:977-993``."""
    m = head_dim // 6
    c = torch.empty(res, m, dtype=torch.float32, device=device)
    s = torch.empty_like(c)
    check(lib().vdit_rope3d_table(res, head_dim, float(base), ptr(c), ptr(s), _s(c)), "rope3d_table")
    return c, s


def precompute_rope_2d_cond(cond_size: int = 64, base: float = 64.0, head_dim: int = 96,
                            device: Optional[torch.device] = None):
    """[cond_size^2, 2, head_dim//4] cos/sin, ``lib/fast_kernels.py:1011-1035``."""
    m = head_dim // 4
    c = torch.empty(cond_size * cond_size, 2, m, dtype=torch.float32, device=device)
    s = torch.empty_like(c)
    check(lib().vdit_rope2d_table(cond_size, head_dim, float(base), ptr(c), ptr(s), _s(c)), "rope2d_table")
    return c, s


# ----------------------------------------------------------------------------- row kernels

def patchify(xt: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """x = xt @ w^T, xt [N,16] fp32, w [D,16] fp32 -> bf16 [N,D]."""
    xt = xt.to(torch.float32).contiguous()
    out = torch.empty(xt.shape[0], w.shape[0], dtype=BF16, device=xt.device)
    check(lib().vdit_patchify(ptr(xt), xt.shape[0], ptr(w), w.shape[0], ptr(out), _s(xt)), "patchify")
    return out


def fast_modulate(x: torch.Tensor, sizes, scale1: torch.Tensor, shift: torch.Tensor,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """LN(x) * scale1 + shift; ``scale1`` is 1 + scale (fp32 [D])."""
    m, d = x.shape
    out = torch.empty_like(x) if out is None else out
    check(lib().vdit_modulate(ptr(x), m, d, ptr(scale1), ptr(shift), ptr(out), _s(x)), "modulate")
    return out


def fast_gate_add_and_modulate(x: torch.Tensor, h: torch.Tensor, gate: torch.Tensor,
                               scale1: Optional[torch.Tensor], shift: Optional[torch.Tensor],
                               out: Optional[torch.Tensor] = None, broadcast_h: bool = False):
    """x += h * gate in place; returns LN(x) * scale1 + shift (or None when scale1 is None).
    ``broadcast_h`` adds one [D] row of h to every row of x."""
    m, d = x.shape
    mod = None
    if scale1 is not None:
        mod = torch.empty_like(x) if out is None else out
    stride = 0 if broadcast_h else h.stride(0)
    check(lib().vdit_gate_add_modulate(ptr(x), ptr(h), stride, m, d, ptr(gate), ptr(scale1), ptr(shift), ptr(mod),
                                       _s(x)), "gate_add_modulate")
    return mod


def fast_gate_add2_and_modulate(x: torch.Tensor, h: torch.Tensor, gate: torch.Tensor, c_row: torch.Tensor,
                                gate2: torch.Tensor, scale1: Optional[torch.Tensor], shift: Optional[torch.Tensor],
                                out: Optional[torch.Tensor] = None):
    """Two gate-adds in one pass: x += h * gate, then x += c_row * gate2 (one [D] row for
    every row), each rounded to bf16 as its own pass would; returns LN(x) * scale1 + shift
    (or None when scale1 is None)."""
    m, d = x.shape
    if c_row.dtype != BF16 or c_row.numel() != d or gate2.numel() != d:
        raise ValueError(f"fast_gate_add2_and_modulate: c_row must be a bf16 row of {d}, gate2 of {d}")
    mod = None
    if scale1 is not None:
        mod = torch.empty_like(x) if out is None else out
    c = c_row.reshape(-1).contiguous()
    g2 = _f32(gate2)
    check(lib().vdit_gate_add2_modulate(ptr(x), ptr(h), h.stride(0), m, d, ptr(gate), ptr(c), ptr(g2), ptr(scale1),
                                        ptr(shift), ptr(mod), _s(x)), "gate_add2_modulate")
    return mod


def fast_gate_add(x: torch.Tensor, h: torch.Tensor, gate: torch.Tensor, broadcast_h: bool = False) -> torch.Tensor:
    fast_gate_add_and_modulate(x, h, gate, None, None, broadcast_h=broadcast_h)
    return x


def fast_out_modulate_unpatchify(x: torch.Tensor, sizes, scale1: torch.Tensor, shift: torch.Tensor,
                                 w_fp32: torch.Tensor) -> torch.Tensor:
    """[N,16] fp32 = bf16(LN(x)*scale1+shift) @ w^T (``lib/fast_kernels.py:888-940``)."""
    m, d = x.shape
    out = torch.empty(m, w_fp32.shape[0], dtype=torch.float32, device=x.device)
    check(lib().vdit_out_modulate_unpatchify(ptr(x), m, d, ptr(scale1), ptr(shift), ptr(w_fp32), ptr(out), _s(x)),
          "out_modulate_unpatchify")
    return out


def split_weight3(w_fp32: torch.Tensor) -> torch.Tensor:
    """[3R, D] bf16 three-part split of an fp32 [R, D] weight (hi, mid, lo row blocks)."""
    r, d = w_fp32.shape
    w3 = torch.empty(3 * r, d, dtype=torch.bfloat16, device=w_fp32.device)
    check(lib().vdit_split_weight3(ptr(w_fp32), r, d, ptr(w3), _s(w_fp32)), "split_weight3")
    return w3


def unpatchify_project(y: torch.Tensor, w3: torch.Tensor) -> torch.Tensor:
    """[N,16] fp32 = y (bf16, already modulated) @ w^T at fp32 accuracy, w as its split ``w3``
    (the projection of ``lib/fast_kernels.py:613-648``)."""
    m, d = y.shape
    out = torch.empty(m, 16, dtype=torch.float32, device=y.device)
    check(lib().vdit_unpatchify_project(ptr(y), m, d, ptr(w3), ptr(out), _s(y)), "unpatchify_project")
    return out


def fused_qknorm_rope3d_gather(qkv: torch.Tensor, q_scale: torch.Tensor, k_scale: torch.Tensor,
                               cos_t: torch.Tensor, sin_t: torch.Tensor, h_coords: torch.Tensor,
                               fwd_idx: Optional[torch.Tensor], heads: int, head_dim: int,
                               out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Hilbert-gathered [N,3,H,HD]: RoPE3D(RMS(q)*qs), RoPE3D(RMS(k)*ks), v
    (``lib/fast_kernels.py:1476-1535``)."""
    n = qkv.shape[0]
    out = torch.empty(n, 3 * heads * head_dim, dtype=BF16, device=qkv.device) if out is None else out
    check(lib().vdit_qknorm_rope3d_gather(ptr(qkv), n, heads, head_dim, ptr(q_scale), ptr(k_scale), ptr(cos_t),
                                          ptr(sin_t), cos_t.shape[0], ptr(h_coords), ptr(fwd_idx), ptr(out), _s(qkv)),
          "qknorm_rope3d_gather")
    return out


def fused_qknorm_rope2d_cond_inplace(qkv: torch.Tensor, q_scale: torch.Tensor, k_scale: torch.Tensor,
                                     cos2d: torch.Tensor, sin2d: torch.Tensor, heads: int, head_dim: int,
                                     n_prefix: int = 5) -> torch.Tensor:
    """Context tokens in place: RMS(q,k)*scale, 2D RoPE on tokens >= 5
    (``lib/fast_kernels.py:1412-1473``)."""
    l = qkv.shape[0]
    need = max(l - n_prefix, 0) * 2 * (head_dim // 4)      # (token, axis) rows x hd/4 frequencies
    if need and (cos2d is None or sin2d is None or cos2d.numel() < need or sin2d.numel() < need):
        raise ValueError(f"2D RoPE tables cover fewer than the {l - n_prefix} rotated context tokens")
    check(lib().vdit_qknorm_rope2d(ptr(qkv), l, heads, head_dim, ptr(q_scale), ptr(k_scale), ptr(cos2d), ptr(sin2d),
                                   n_prefix, _s(qkv)), "qknorm_rope2d")
    return qkv


def vec_ln_modulate(v: torch.Tensor, scale1: torch.Tensor, shift: torch.Tensor) -> torch.Tensor:
    """bf16 LN(v) * scale1 + shift of one fp32 [D] vector (the 1-token context stream)."""
    v = v.reshape(-1)
    out = torch.empty(v.numel(), dtype=BF16, device=v.device)
    check(lib().vdit_vec_ln_modulate(ptr(v), v.numel(), ptr(scale1), ptr(shift), ptr(out), _s(v)), "vec_ln_modulate")
    return out


def vec_gate_residual_(c: torch.Tensor, y: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
    """c += float(y) * gate in place (fp32 [D] vector, bf16 update)."""
    check(lib().vdit_vec_gate_residual(ptr(c), ptr(y.reshape(-1)), ptr(gate), c.numel(), _s(c)), "vec_gate_residual")
    return c


def fast_swiglu_from_packed(h_packed: torch.Tensor) -> torch.Tensor:
    """silu(h[:, F:]) * h[:, :F] (``lib/fast_kernels.py:942-974``)."""
    m, f2 = h_packed.shape
    out = torch.empty(m, f2 // 2, dtype=BF16, device=h_packed.device)
    check(lib().vdit_swiglu_packed(ptr(h_packed), m, f2 // 2, ptr(out), _s(h_packed)), "swiglu_packed")
    return out


def build_conv_plan(conv_indices, row_order: torch.Tensor) -> torch.Tensor:
    """Shared-memory staging plan for the fused conv + SwiGLU, built once per
    voxel set from the conv index table (``build_conv_indices_fast``) and a
    Hilbert order of the rows; see ``fast_sparse_conv3d_swiglu_planned``."""
    idx = conv_indices[0] if isinstance(conv_indices, (list, tuple)) else conv_indices
    n = idx.shape[0]
    order = row_order.to(torch.int64).contiguous()
    plan = torch.empty(max(1, int(lib().vdit_dwconv27_plan_bytes(n))), dtype=torch.uint8, device=idx.device)
    check(lib().vdit_dwconv27_plan(ptr(idx), ptr(order), n, ptr(plan), plan.numel(), _s(idx)), "dwconv27_plan")
    return plan


def fast_sparse_conv3d_swiglu_planned(feat: torch.Tensor, weight_fp32: torch.Tensor, bias_fp32: torch.Tensor,
                                      plan: torch.Tensor, bf16_weights: bool = False) -> torch.Tensor:
    """silu(conv(feat)[:, C/2:]) * conv(feat)[:, :C/2] from a ``build_conv_plan``, with
    ``feat``, ``weight_fp32`` and ``bias_fp32`` in pair-interleaved column order
    (a[2k], a[2k+1], gate[2k], gate[2k+1]); bit-identical to
    ``fast_sparse_conv3d(..., fuse_swiglu=True)`` on the de-interleaved inputs.
    ``bf16_weights``: the weights hold bf16 values (``weights_are_bf16``); the faster
    bf16-operand FMAs then give the same bits."""
    n, c = feat.shape
    out = torch.empty(n, c // 2, dtype=BF16, device=feat.device)
    fn = lib().vdit_dwconv27_swiglu_planned_bf16w if bf16_weights else lib().vdit_dwconv27_swiglu_planned
    check(fn(ptr(feat), n, c, ptr(plan), ptr(weight_fp32), ptr(bias_fp32), ptr(out), _s(feat)),
          "dwconv27_swiglu_planned")
    return out


def weights_are_bf16(w: torch.Tensor) -> bool:
    """True when every value of the fp32 tensor is exactly a bf16 value (one check per
    weight set; it selects the bf16-operand conv)."""
    return bool((w.to(BF16).to(torch.float32) == w).all())


def fast_sparse_conv3d(feat: torch.Tensor, weight_fp32: torch.Tensor, bias_fp32: torch.Tensor,
                       conv_indices, fuse_swiglu: bool = False) -> torch.Tensor:
    """Depthwise 27-tap conv (``lib/fast_kernels.py:1704-1736``); with
    ``fuse_swiglu`` returns silu(y[:, C/2:]) * y[:, :C/2]."""
    idx = conv_indices[0] if isinstance(conv_indices, (list, tuple)) else conv_indices
    n, c = feat.shape
    out = torch.empty(n, c // 2 if fuse_swiglu else c, dtype=BF16, device=feat.device)
    check(lib().vdit_dwconv27(ptr(feat), n, c, ptr(idx), ptr(weight_fp32), ptr(bias_fp32), ptr(out),
                              1 if fuse_swiglu else 0, _s(feat)), "dwconv27")
    return out


def dense_sparse_conv3d(feat: torch.Tensor, weight_t_bf16: torch.Tensor, bias_fp32: torch.Tensor,
                        conv_indices) -> torch.Tensor:
    """Dense 27-tap sparse conv (``BK/ops/sparse.py:84-123``); ``weight_t_bf16`` is
    [27, C_out, C_in] (the reference (3,3,3,C_in,C_out) weight transposed)."""
    idx = conv_indices[0] if isinstance(conv_indices, (list, tuple)) else conv_indices
    n, cin = feat.shape
    cout = weight_t_bf16.shape[1]
    out = torch.empty(n, cout, dtype=BF16, device=feat.device)
    check(lib().vdit_dense_conv27(ptr(feat), n, cin, cout, ptr(idx), ptr(weight_t_bf16), ptr(bias_fp32), ptr(out),
                                  _s(feat)), "dense_conv27")
    return out


# ----------------------------------------------------------------------------- linears

def linear(a: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None,
           out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``F.linear(a, w, bias)`` for bf16 2D ``a`` [M, K] (row stride free) and a
    contiguous bf16 weight [N, K] on the tcgen05 GEMM (N and K multiples of 8)."""
    if a.dtype != BF16 or w.dtype != BF16 or a.dim() != 2 or w.dim() != 2 or a.shape[1] != w.shape[1]:
        raise ValueError(f"linear: a {tuple(a.shape)} {a.dtype} and w {tuple(w.shape)} {w.dtype} "
                         "must be 2D bf16 with the same K")
    if a.stride(1) != 1 or w.stride(1) != 1:
        raise ValueError("linear: a and w need unit column stride")
    m, k = a.shape
    n = w.shape[0]
    if bias is not None and (bias.dtype != BF16 or bias.numel() != n or not bias.is_contiguous()):
        raise ValueError(f"linear: bias must be a contiguous bf16 vector of {n}")
    if out is None:
        out = torch.empty(m, n, dtype=BF16, device=a.device)
    elif out.dtype != BF16 or out.dim() != 2 or out.shape[0] < m or out.shape[1] < n or out.stride(1) != 1:
        raise ValueError(f"linear: out must be a bf16 2D view of at least [{m}, {n}]")
    check(lib().vdit_linear(ptr(a), a.stride(0), ptr(w), w.stride(0), ptr(bias), ptr(out), out.stride(0), m, n, k,
                            _s(a)), "linear")
    return out


GEMV_X_BF16, GEMV_X_F32, GEMV_X_LN_MOD, GEMV_X_SWIGLU = 0, 1, 2, 3


def gemv(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None, *, x_mode: Optional[int] = None,
         mod_scale: Optional[torch.Tensor] = None, mod_shift: Optional[torch.Tensor] = None,
         out_dtype: torch.dtype = BF16, silu_out: bool = False) -> torch.Tensor:
    """One-row linear(s) ``act(W x' + b)`` on the GEMV kernel.  ``w`` is [n, k] or a batch
    [B, n, k] (bf16 or fp32, contiguous), ``bias`` [n] / [B, n] of ``w``'s dtype.  ``x'`` is
    formed from ``x`` by the prologue ``x_mode`` (default: the plain vector of ``x``'s dtype):
    ``GEMV_X_LN_MOD`` = bf16(LN(x) * mod_scale + mod_shift) of an fp32 [k] vector (per-batch
    ``mod_scale``/``mod_shift`` as [B, k] views), ``GEMV_X_SWIGLU`` = bf16(silu(g) * a) of a
    bf16 [2k] vector [a | g].  Returns [n] or [B, n] in ``out_dtype`` (bf16 or fp32)."""
    batched = w.dim() == 3
    wb = w if batched else w.unsqueeze(0)
    B, n, k = wb.shape
    if w.dtype not in (BF16, torch.float32) or not wb.is_contiguous():
        raise ValueError("gemv: w must be contiguous bf16 or fp32 [n, k] or [B, n, k]")
    if bias is not None and (bias.dtype != w.dtype or bias.numel() != B * n or not bias.is_contiguous()):
        raise ValueError(f"gemv: bias must be contiguous {w.dtype} with {B * n} elements")
    if x_mode is None:
        x_mode = GEMV_X_F32 if x.dtype == torch.float32 else GEMV_X_BF16
    want = {GEMV_X_BF16: (BF16, k), GEMV_X_F32: (torch.float32, k), GEMV_X_LN_MOD: (torch.float32, k),
            GEMV_X_SWIGLU: (BF16, 2 * k)}[x_mode]
    if x.dtype != want[0] or x.stride(-1) != 1 or x.shape[-1] != want[1]:
        raise ValueError(f"gemv: x must be {want[0]} with {want[1]} elements per vector (mode {x_mode})")
    x_bs = x.stride(0) if x.dim() == 2 else 0
    if x.dim() == 2 and x.shape[0] != B:
        raise ValueError("gemv: a batch of inputs needs one vector per weight matrix")
    mod_bs = 0
    if x_mode == GEMV_X_LN_MOD:
        if mod_scale is None or mod_shift is None:
            raise ValueError("gemv: GEMV_X_LN_MOD needs mod_scale and mod_shift")
        for t in (mod_scale, mod_shift):
            if t.dtype != torch.float32 or t.stride(-1) != 1 or t.shape[-1] != k:
                raise ValueError("gemv: mod_scale / mod_shift must be fp32 with unit stride and k columns")
        if mod_scale.dim() == 2:
            if mod_scale.shape[0] != B or mod_scale.stride(0) != mod_shift.stride(0):
                raise ValueError("gemv: per-batch mod_scale / mod_shift need one row per entry and one stride")
            mod_bs = mod_scale.stride(0)
    if out_dtype not in (BF16, torch.float32):
        raise ValueError("gemv: out_dtype must be bf16 or fp32")
    out = torch.empty(B, n, dtype=out_dtype, device=w.device)
    check(lib().vdit_gemv(x_mode, ptr(x), x_bs, ptr(mod_scale), ptr(mod_shift), mod_bs, int(w.dtype == torch.float32),
                          ptr(wb), n * k, ptr(bias), n, int(out_dtype == torch.float32), int(silu_out), ptr(out), n,
                          n, k, B, _s(w)), "gemv")
    return out if batched else out[0]


def linear_qkv_rope3d(a: torch.Tensor, w: torch.Tensor, bias: torch.Tensor, q_scale: torch.Tensor,
                      k_scale: torch.Tensor, cos_t: torch.Tensor, sin_t: torch.Tensor, h_coords: torch.Tensor,
                      bwd_idx: torch.Tensor, heads: int, head_dim: int,
                      out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``fused_qknorm_rope3d_gather(F.linear(a, w, bias), ..., fwd)`` in one tcgen05 GEMM:
    the QK-norm / RoPE3D pass runs in the GEMM epilogue and input row r is written to
    row ``bwd_idx[r]`` (``bwd_idx`` = the inverse of the window order ``fwd``)."""
    m, k = a.shape
    n = 3 * heads * head_dim
    if a.dtype != BF16 or w.dtype != BF16 or bias.dtype != BF16 or a.stride(1) != 1 or w.shape != (n, k) \
            or not w.is_contiguous() or bias.numel() != n:
        raise ValueError("linear_qkv_rope3d: bf16 a [M, K] (unit column stride), w [3*H*HD, K], bias [3*H*HD]")
    if h_coords.dtype != torch.int32 or h_coords.shape != (m, 4) or not h_coords.is_contiguous():
        raise ValueError("linear_qkv_rope3d: h_coords must be contiguous int32 [M, 4]")
    if bwd_idx.dtype != torch.int64 or bwd_idx.numel() != m:
        raise ValueError("linear_qkv_rope3d: bwd_idx must be int64 [M]")
    for t in (q_scale, k_scale, cos_t, sin_t):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError("linear_qkv_rope3d: scales and RoPE tables must be contiguous fp32")
    if out is None:
        out = torch.empty(m, n, dtype=BF16, device=a.device)
    check(lib().vdit_linear_qkv_rope3d(ptr(a), a.stride(0), ptr(w), w.stride(0), ptr(bias), ptr(q_scale),
                                       ptr(k_scale), ptr(cos_t), ptr(sin_t), cos_t.shape[0], ptr(h_coords),
                                       ptr(bwd_idx), ptr(out), out.stride(0), m, heads, head_dim, k, _s(a)),
          "linear_qkv_rope3d")
    return out


# ----------------------------------------------------------------------------- attention

def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_q: Sequence[int], cu_k: Sequence[int],
              heads: int, head_dim: int, out: Optional[torch.Tensor] = None,
              out_rows: Optional[torch.Tensor] = None, scale: Optional[float] = None) -> torch.Tensor:
    """Varlen non-causal attention on tcgen05.  q/k/v are 2D views [rows, >=H*HD]
    (any row stride); ``cu_q``/``cu_k`` are host lists of segment offsets;
    ``out_rows`` scatters output row i to out_rows[i]."""
    if out is None:
        out = torch.empty(q.shape[0], heads * head_dim, dtype=BF16, device=q.device)
    for t, name in ((q, "q"), (k, "k"), (v, "v"), (out, "out")):
        if t.dtype != BF16 or t.dim() != 2:
            raise ValueError(f"attention: {name} must be a 2D bf16 view, got {tuple(t.shape)} {t.dtype}")
    if len(cu_q) != len(cu_k) or len(cu_q) < 2:
        raise ValueError("attention: cu_q and cu_k need the same number (>= 2) of offsets")
    # the kernel reads rows [0, cu[-1]) through tensor maps built from these offsets
    if int(cu_q[-1]) > q.shape[0] or int(cu_k[-1]) > k.shape[0] or int(cu_k[-1]) > v.shape[0]:
        raise ValueError(f"attention: offsets end at {int(cu_q[-1])}/{int(cu_k[-1])} rows, past q/k/v "
                         f"of {q.shape[0]}/{k.shape[0]}/{v.shape[0]} rows")
    if out_rows is None and int(cu_q[-1]) > out.shape[0]:
        raise ValueError(f"attention: out has {out.shape[0]} rows, fewer than the {int(cu_q[-1])} query rows")
    if out_rows is not None and out_rows.dtype != torch.int64:
        raise ValueError(f"attention: out_rows must be int64, got {out_rows.dtype}")
    if out_rows is not None and out_rows.numel() < int(cu_q[-1]):
        raise ValueError(f"attention: out_rows has {out_rows.numel()} entries for {int(cu_q[-1])} query rows")
    nseg = len(cu_q) - 1
    cq, ck = _host_i32(cu_q), _host_i32(cu_k)      # host arrays, alive for the call
    scale = 1.0 / math.sqrt(head_dim) if scale is None else scale
    check(lib().vdit_attention(ptr(q), q.stride(0), ptr(k), k.stride(0), ptr(v), v.stride(0), ptr(out), out.stride(0),
                               ptr(out_rows), ctypes.addressof(cq), ctypes.addressof(ck), nseg, heads, head_dim,
                               float(scale), _s(q)), "attention")
    return out


def _host_i32(vals: Sequence[int]):
    return (ctypes.c_int32 * len(vals))(*[int(v) for v in vals])


def flash_varlen_qkvpacked_already_sorted(qkv_sorted: torch.Tensor, cu_seqlens, max_len: int, heads: int,
                                          head_dim: int, out_rows: Optional[torch.Tensor] = None,
                                          out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Window self-attention over Hilbert-sorted packed qkv [N, 3*H*HD]
    (``lib/fast_kernels.py:1538-1587``); ``out_rows`` = fwd index scatters the
    result back to voxel order (fusing ``out[bwd_idx]``)."""
    d = heads * head_dim
    cu = getattr(cu_seqlens, "host", None) or [int(v) for v in cu_seqlens.tolist()]
    return attention(qkv_sorted[:, :d], qkv_sorted[:, d:2 * d], qkv_sorted[:, 2 * d:], cu, cu, heads, head_dim,
                     out=out, out_rows=out_rows)


def flash_cross_attn(q: torch.Tensor, cu_q, max_q: int, kv: torch.Tensor, cu_k, max_k: int, heads: int,
                     head_dim: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Cross attention, q [Nq, H*HD], kv [Nk, 2*H*HD] packed (``lib/fast_kernels.py:1605-1646``)."""
    d = heads * head_dim
    cq = getattr(cu_q, "host", None) or [int(v) for v in (cu_q.tolist() if torch.is_tensor(cu_q) else cu_q)]
    ck = getattr(cu_k, "host", None) or [int(v) for v in (cu_k.tolist() if torch.is_tensor(cu_k) else cu_k)]
    return attention(q, kv[:, :d], kv[:, d:2 * d], cq, ck, heads, head_dim, out=out)


def flash_cond_self_attn(qkv_cond: torch.Tensor, heads: int, head_dim: int,
                         out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Full self-attention over the context tokens, packed [L, 3*H*HD]
    (``lib/fast_kernels.py:1590-1602``)."""
    d = heads * head_dim
    l = qkv_cond.shape[0]
    return attention(qkv_cond[:, :d], qkv_cond[:, d:2 * d], qkv_cond[:, 2 * d:], [0, l], [0, l], heads, head_dim,
                     out=out)


def attention_1q(q: torch.Tensor, kv: torch.Tensor, heads: int, head_dim: int,
                 k_offset: int = 0, v_offset: Optional[int] = None) -> torch.Tensor:
    """One query per head ([H*HD]) over the rows of ``kv`` (K at column
    ``k_offset``, V at ``v_offset``): the 1-token context->x attention
    (``lib/fast_flow.py:1769-1777``)."""
    d = heads * head_dim
    v_offset = k_offset + d if v_offset is None else v_offset
    if kv.dtype != BF16 or kv.dim() != 2 or q.numel() != d:
        raise ValueError(f"attention_1q: kv must be 2D bf16 and q hold {d} values")
    if min(k_offset, v_offset) < 0 or max(k_offset, v_offset) + d > kv.shape[1]:
        raise ValueError(f"attention_1q: K/V columns at {k_offset}/{v_offset} run past the {kv.shape[1]} of kv")
    n = kv.shape[0]
    ws = torch.empty(int(lib().vdit_attention_1q_workspace_bytes(heads, head_dim, n)), dtype=torch.uint8,
                     device=kv.device)
    out = torch.empty(d, dtype=BF16, device=kv.device)
    q = q.reshape(-1).to(BF16).contiguous()
    check(lib().vdit_attention_1q(ptr(q), ptr(kv[:, k_offset:]), ptr(kv[:, v_offset:]), kv.stride(0), n, heads,
                                  head_dim, float(1.0 / math.sqrt(head_dim)), ptr(out), ptr(ws), ws.numel(), _s(kv)),
          "attention_1q")
    return out


def attention_1q_wide(q: torch.Tensor, x: torch.Tensor, w_kv: torch.Tensor, b_kv: torch.Tensor, heads: int,
                      head_dim: int) -> torch.Tensor:
    """One query per head ([H*HD]) over keys K = x W_k^T + b_k and values V = x W_v^T + b_v
    (``w_kv`` = [W_k; W_v] [2D, D], ``b_kv`` = [b_k; b_v]) without forming K and V: the
    1-token context->x attention (``lib/fast_flow.py:1769-1777``) on the voxel rows x."""
    d = heads * head_dim
    if x.dtype != BF16 or x.dim() != 2 or x.shape[1] != d or x.stride(1) != 1:
        raise ValueError(f"attention_1q_wide: x must be a bf16 [n, {d}] view")
    if w_kv.dtype != BF16 or w_kv.shape != (2 * d, d) or not w_kv.is_contiguous() or b_kv.numel() != 2 * d:
        raise ValueError(f"attention_1q_wide: w_kv must be contiguous bf16 [{2 * d}, {d}], b_kv [{2 * d}]")
    n = x.shape[0]
    ws = torch.empty(int(lib().vdit_attention_1q_wide_workspace_bytes(heads, head_dim, n)), dtype=torch.uint8,
                     device=x.device)
    out = torch.empty(d, dtype=BF16, device=x.device)
    q = q.reshape(-1).to(BF16).contiguous()
    bv = b_kv.reshape(-1)[d:].to(BF16).contiguous()
    check(lib().vdit_attention_1q_wide(ptr(q), ptr(x), x.stride(0), n, ptr(w_kv[:d]), ptr(w_kv[d:]), w_kv.stride(0),
                                       ptr(bv), heads, head_dim, float(1.0 / math.sqrt(head_dim)), ptr(out), ptr(ws),
                                       ws.numel(), _s(x)), "attention_1q_wide")
    return out


# ----------------------------------------------------------------------------- sampler glue

def gather_rows_f32(src: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    src = src.to(torch.float32).contiguous()
    out = torch.empty(idx.shape[0], src.shape[1], dtype=torch.float32, device=src.device)
    check(lib().vdit_gather_rows_f32(ptr(src), ptr(idx), idx.shape[0], src.shape[1], ptr(out), _s(src)), "gather_rows")
    return out


def cfg_euler_(xt: torch.Tensor, v_pos: torch.Tensor, v_neg: Optional[torch.Tensor], guidance: float, dt: float):
    check(lib().vdit_cfg_euler(ptr(xt), ptr(v_pos), ptr(v_neg), xt.shape[0], float(guidance), float(dt), _s(xt)),
          "cfg_euler")
    return xt


def cfg_reuse_euler_(xt: torch.Tensor, v_pos: torch.Tensor, last_neg: torch.Tensor,
                     last_neg_x0: Optional[torch.Tensor], guidance: float, dt: float, t_eval: float,
                     endpoint_blend: float, hf_gain: float, zero_star: bool) -> torch.Tensor:
    """Euler step of a guided step that reuses the last unconditional velocity (the
    reference's approximate ``neg_reuse`` CFG cache, ``lib/fast_flow.py:2844-2887``): CFG-Zero*
    projection, clean-endpoint blend (``last_neg_x0``, None to skip it) and high-frequency
    boost; xt [N, 16] fp32 updated in place."""
    for t, name in ((xt, "xt"), (v_pos, "v_pos"), (last_neg, "last_neg"), (last_neg_x0, "last_neg_x0")):
        if t is not None and (t.dtype != torch.float32 or t.shape != xt.shape or not t.is_contiguous()):
            raise ValueError(f"cfg_reuse_euler_: {name} must be contiguous fp32 {tuple(xt.shape)}")
    ws = torch.empty(int(lib().vdit_cfg_reuse_workspace_bytes()), dtype=torch.uint8, device=xt.device)
    check(lib().vdit_cfg_reuse_euler(ptr(xt), ptr(v_pos), ptr(last_neg), ptr(last_neg_x0), xt.shape[0],
                                     float(guidance), float(dt), float(t_eval), float(endpoint_blend), float(hf_gain),
                                     int(bool(zero_star)), ptr(ws), ws.numel(), _s(xt)), "cfg_reuse_euler")
    return xt


def neg_endpoint(xt: torch.Tensor, v_neg: torch.Tensor, t_eval: float) -> torch.Tensor:
    """x0 = xt - t_eval * v_neg ([N, 16] fp32): the clean endpoint the CFG cache blends toward."""
    out = torch.empty_like(xt)
    check(lib().vdit_neg_endpoint(ptr(xt), ptr(v_neg), xt.shape[0], float(t_eval), ptr(out), _s(xt)), "neg_endpoint")
    return out


def unpermute_denorm(xt: torch.Tensor, up_widx: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor) -> torch.Tensor:
    out = torch.empty_like(xt)
    check(lib().vdit_unpermute_denorm(ptr(xt), ptr(up_widx), xt.shape[0], ptr(scale), ptr(shift), ptr(out), _s(xt)),
          "unpermute_denorm")
    return out
