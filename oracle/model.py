"""torch-fp32 CPU restatement of the lat_dit forward path (test oracle only).

Restates ``FlowModel.forward`` (``BK/models/generators/lat_dit.py:743-824``)
with its ``SparseTransformerBlock`` (``:260-585``), the exact 1-token
unconditional condensation of ``lib/fast_flow.py`` (``:195-309, 937-958,
1702-1794, 2295-2309``), the depthwise and dense 27-tap sparse convolutions
(``BK/ops/libsparse/conv.cu:187-309, 468-494``) and the exact Euler+CFG
sampler (``BK/kandi3d_image23d/modules/lat_dit/core.py:114-177`` with the
piecewise schedule of ``lib/fast_sampler.py:670-732``).  ``BK/`` abbreviates
``baseline_repo/3dgen-main/``.

Parameters are a flat dict keyed by the reference checkpoint names
(``flow.blocks.{i}.to_qkv.weight`` ...), all fp32 on CPU.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np
import torch
import torch.nn.functional as F

from . import geometry as geo

Params = Dict[str, torch.Tensor]


@dataclass
class ModelConfig:
    """Architecture of ``FlowModel`` as used by the lat_dit checkpoint
    (``weights/config.json``: dim 1536, head_dim 96, depth 24, cond_depth 8,
    ffn_rate 2.5, res 64, orders h/ht1/h1/ht, patch_size 4096)."""
    dim: int = 1536
    head_dim: int = 96
    depth: int = 24
    cond_depth: int = 8
    ffn_rate: float = 2.5
    res: int = 64
    latent_dim: int = 16
    time_pos_features: int = 256
    patch_size: int = 4096
    dino_dim: int = 1280
    latent_scale: float = 1.5
    orders: tuple = geo.ORDERS

    @property
    def heads(self) -> int:
        return self.dim // self.head_dim

    @property
    def ffn_dim(self) -> int:
        return int(self.dim * self.ffn_rate)


def param_shapes(cfg: ModelConfig) -> Dict[str, tuple]:
    """Checkpoint key -> shape, as in the lat_dit safetensors header."""
    D, F2, Fh, L = cfg.dim, 2 * cfg.ffn_dim, cfg.ffn_dim, cfg.latent_dim
    H, HD = cfg.heads, cfg.head_dim
    s = {
        "image_map.weight": (D, cfg.dino_dim), "image_map.bias": (D,),
        "flow.time_embed.0.weight": (4 * D, cfg.time_pos_features), "flow.time_embed.0.bias": (4 * D,),
        "flow.time_embed.2.weight": (D, 4 * D), "flow.time_embed.2.bias": (D,),
        "flow.patchify.weight": (D, L), "flow.unpatchify.weight": (L, D),
        "flow.out_gates.weight": (2 * D, D), "flow.out_gates.bias": (2 * D,),
        "mean": (L,), "std": (L,),
    }
    for b in range(cfg.depth):
        p = f"flow.blocks.{b}."
        lin = {"gates": (9 * D, D), "to_qkv": (3 * D, D), "to_out": (D, D),
               "to_out_cross": (D, D), "ffn0": (F2, D), "ffn1": (D, Fh)}
        if b < cfg.cond_depth:
            lin.update({"cond_gates": (9 * D, D), "cond_to_qkv": (3 * D, D), "cond_to_out": (D, D),
                        "to_qkv_cross": (3 * D, D), "cond_to_qkv_cross": (3 * D, D),
                        "cond_to_out_cross": (D, D), "cond_ffn0": (F2, D), "cond_ffn1": (D, Fh)})
        else:
            lin.update({"to_q_cross": (D, D), "cond_gates": (2 * D, D), "cond_to_kv_cross": (2 * D, D)})
        for n, sh in lin.items():
            s[p + n + ".weight"] = sh
            s[p + n + ".bias"] = (sh[0],)
        s[p + "ffn_conv.weight"] = (3, 3, 3, F2)
        s[p + "ffn_conv.bias"] = (F2,)
        s[p + "qk_norm.q_scale"] = (H, HD)
        s[p + "qk_norm.k_scale"] = (H, HD)
        if b < cfg.cond_depth:
            s[p + "cond_qk_norm.q_scale"] = (H, HD)
            s[p + "cond_qk_norm.k_scale"] = (H, HD)
    return s


def init_params(cfg: ModelConfig, seed: int, weight_std: float = 0.02, bias_std: float = 0.0,
                scale_jitter: float = 0.0) -> Params:
    """Seeded random-init weights: linears N(0, weight_std), biases N(0, bias_std),
    q/k RMSNorm gains 1 (+ N(0, scale_jitter)), conv weights N(0, weight_std),
    mean 0 / std 1.  Keys are drawn in sorted order from one CPU generator so
    the same seed reproduces the same tensors everywhere."""
    g = torch.Generator().manual_seed(seed)
    out: Params = {}
    for k, sh in sorted(param_shapes(cfg).items()):
        if k == "mean":
            t = torch.zeros(sh)
        elif k == "std":
            t = torch.ones(sh)
        elif k.endswith("_scale"):
            t = 1.0 + scale_jitter * torch.randn(sh, generator=g)
        elif k.endswith(".bias"):
            t = bias_std * torch.randn(sh, generator=g)
        else:
            t = weight_std * torch.randn(sh, generator=g)
        out[k] = t.float().contiguous()
    return out


# ----------------------------------------------------------------------------- primitives

def time_encoding(t: torch.Tensor, dim: int, max_period: float = 10000.0) -> torch.Tensor:
    """``BK/base_models/fourier_utils.py:33-44`` (fp64 frequencies, [cos, sin])."""
    omega = torch.exp(-math.log(max_period) * torch.arange(0, dim, 2, dtype=torch.float64) / dim)
    f = t.to(torch.float64)[..., None] * omega
    return torch.cat([torch.cos(f), torch.sin(f)], -1).float()


def layer_norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """LayerNorm without affine, eps 1e-6 (``lat_dit.py:19-23``)."""
    mu = x.mean(-1, keepdim=True)
    var = ((x - mu) ** 2).mean(-1, keepdim=True)
    return (x - mu) * torch.rsqrt(var + eps)


def modulate(x, scale, shift):
    """``lat_dit.py:63-66``: LN(x) * (1 + scale) + shift."""
    return layer_norm(x) * (1 + scale) + shift


def rms_norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + eps)


def rope_nd(x: torch.Tensor, pos: torch.Tensor, base: float) -> torch.Tensor:
    """N-d RoPE on [..., H, K] with pos [..., P]; ``lib/fast_kernels.py:316-333``
    (== ``BK/ops/curope/rope.cu:17-89`` when K % (2P) == 0).  Channels
    [2Md, 2Md+M) rotate with [2Md+M, 2M(d+1)); leftover channels pass through."""
    K = x.shape[-1]
    P = pos.shape[-1]
    M = K // (2 * P)
    inv = float(base) ** (-torch.arange(M, dtype=torch.float64) / float(M))
    outs = []
    for d in range(P):
        ang = pos[..., d:d + 1].to(torch.float64) * inv
        c = torch.cos(ang).float().unsqueeze(-2)
        s = torch.sin(ang).float().unsqueeze(-2)
        u = x[..., d * 2 * M: d * 2 * M + M]
        v = x[..., d * 2 * M + M: (d + 1) * 2 * M]
        outs += [u * c - v * s, u * s + v * c]
    if 2 * P * M < K:
        outs.append(x[..., 2 * P * M:])
    return torch.cat(outs, -1)


def attention(q, k, v, score_bytes: int = 1 << 28):
    """softmax(q k^T / sqrt(HD)) v on [n, H, HD] (flash-attn default scale).  Query rows are
    taken in chunks whose fp32 score block stays under ``score_bytes`` (each row's softmax is
    independent, so chunking changes no result beyond matmul rounding); without it a
    16384 x 4101 cross-attention would hold several 3.2 GB score temporaries."""
    nq, nk, heads = q.shape[0], k.shape[0], q.shape[1]
    step = max(1, score_bytes // max(1, 4 * heads * nk))
    if step >= nq:
        s = torch.einsum("qhd,khd->hqk", q, k) / math.sqrt(q.shape[-1])
        return torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v)
    return torch.cat([attention(q[i:i + step], k, v, score_bytes) for i in range(0, nq, step)])


def dwconv27(h: torch.Tensor, w: torch.Tensor, b: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    """Depthwise 27-tap submanifold conv, ``BK/ops/libsparse/conv.cu:187-309``:
    out[n,c] = b[c] + sum_d w[d,c] * h[idx[n,d], c] (fp32 accumulate)."""
    w = w.reshape(27, -1)
    out = b.float().expand(h.shape[0], -1).clone()
    hf = h.float()
    for d in range(27):
        sel = idx[:, d] >= 0
        out[sel] += hf[idx[sel, d].long()] * w[d]
    return out


def dense_conv27(f: torch.Tensor, w: torch.Tensor, b: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    """Dense 27-tap sparse conv, ``BK/ops/libsparse/conv.cu:468-494`` with weight
    (3,3,3,C_in,C_out): out[n,co] = b[co] + sum_d sum_ci W[d,ci,co] f[idx[n,d],ci]."""
    w = w.reshape(27, f.shape[1], -1).float()
    out = b.float().expand(f.shape[0], -1).clone()
    ff = f.float()
    for d in range(27):
        sel = idx[:, d] >= 0
        if sel.any():
            out[sel] += ff[idx[sel, d].long()] @ w[d]
    return out


def linear(p: Params, name: str, x: torch.Tensor) -> torch.Tensor:
    return F.linear(x, p[name + ".weight"], p.get(name + ".bias"))


# ----------------------------------------------------------------------------- geometry

@dataclass
class Geometry:
    """Static per-sample tensors (cf. ``_prepare_sample_geometry``)."""
    perm: torch.Tensor
    up_widx: torch.Tensor
    h_coords: torch.Tensor
    pos3: torch.Tensor                     # [N,3] fp32 RoPE positions
    orders: List[tuple] = field(default_factory=list)   # (fwd, bwd) per order
    cu_seqlens: List[int] = field(default_factory=list)
    conv_indices: torch.Tensor = None


def build_geometry(vox: np.ndarray, cfg: ModelConfig) -> Geometry:
    g = geo.sample_geometry(vox, cfg.patch_size)
    hc = torch.from_numpy(g["h_coords"])
    pos = (hc[:, 1:].float() + 0.5) / cfg.res * 2 - 1          # lat_dit.py:788-790
    return Geometry(
        perm=torch.from_numpy(g["perm"]), up_widx=torch.from_numpy(g["up_widx"]), h_coords=hc,
        pos3=pos, orders=[(torch.from_numpy(f), torch.from_numpy(b)) for f, b in g["order_caches"]],
        cu_seqlens=[int(v) for v in g["cu_seqlens"]],
        conv_indices=torch.from_numpy(g["conv_indices"]),
    )


def cond_positions(L: int) -> torch.Tensor:
    """2D positions of the image tokens 5..L-1 (``lat_dit.py:543-555``)."""
    s = int(round(math.sqrt(L - 5)))
    assert s * s == L - 5, L
    ii, jj = torch.meshgrid(torch.arange(s), torch.arange(s), indexing="ij")
    pos = torch.stack([ii, jj], -1).view(-1, 2).float()
    return (pos + 0.5) / s * 2 - 1


# ----------------------------------------------------------------------------- model

def time_gates(p: Params, cfg: ModelConfig, t_val: float) -> dict:
    """clf = silu(time_embed(enc(t*1000))) and the per-block gate vectors
    (``lat_dit.py:747-750, 391-392, 409-410, 463-464, 817``); use_token=false
    so the clf token is zero (``core.py:101-109``)."""
    t = torch.tensor([float(t_val) * 1000.0], dtype=torch.float32)
    h = linear(p, "flow.time_embed.0", time_encoding(t, cfg.time_pos_features))
    temb = linear(p, "flow.time_embed.2", F.silu(h))
    clf = F.silu(temb)
    out = {"clf": clf, "blocks": [], "cond": []}
    for b in range(cfg.depth):
        pre = f"flow.blocks.{b}."
        out["blocks"].append(linear(p, pre + "gates", clf).view(9, cfg.dim))
        n = 9 if b < cfg.cond_depth else 2
        out["cond"].append(linear(p, pre + "cond_gates", clf).view(n, cfg.dim))
    out["out"] = linear(p, "flow.out_gates", clf).view(2, cfg.dim)
    return out


def _qknorm(p, pre, q, k):
    """QKNorm: rms_norm(.) * scale, no +1 (``lat_dit.py:241-250``)."""
    return rms_norm(q) * p[pre + "q_scale"], rms_norm(k) * p[pre + "k_scale"]


def block_forward(p: Params, cfg: ModelConfig, b: int, x: torch.Tensor, c: torch.Tensor,
                  gates: dict, geom: Geometry, cpos: Optional[torch.Tensor]):
    """One ``SparseTransformerBlock.__forward`` (``lat_dit.py:364-485``).
    x [N,D] in lexicographic order, c [L,D] context (any L).  Returns (x, c)."""
    H, HD, D = cfg.heads, cfg.head_dim, cfg.dim
    pre = f"flow.blocks.{b}."
    s_msa, sh_msa, g_msa, s_cr, sh_cr, g_cr, s_mlp, sh_mlp, g_mlp = gates["blocks"][b]
    N = x.shape[0]

    # window self-attention in Hilbert order orders[b % 4]
    qkv = linear(p, pre + "to_qkv", modulate(x, s_msa, sh_msa)).view(N, 3, H, HD)
    q, k = _qknorm(p, pre + "qk_norm.", qkv[:, 0], qkv[:, 1])
    q, k = rope_nd(q, geom.pos3, 128.0), rope_nd(k, geom.pos3, 128.0)
    v = qkv[:, 2]
    fwd, bwd = geom.orders[b % len(geom.orders)]
    qs, ks, vs = q[fwd], k[fwd], v[fwd]
    o = torch.empty_like(qs)
    cu = geom.cu_seqlens
    for i in range(len(cu) - 1):
        o[cu[i]:cu[i + 1]] = attention(qs[cu[i]:cu[i + 1]], ks[cu[i]:cu[i + 1]], vs[cu[i]:cu[i + 1]])
    o = o[bwd].reshape(N, D)
    x = x + linear(p, pre + "to_out", o) * g_msa

    if b < cfg.cond_depth:
        cs_msa, csh_msa, cg_msa, cs_cr, csh_cr, cg_cr, cs_mlp, csh_mlp, cg_mlp = gates["cond"][b]
        L = c.shape[0]
        qkvc = linear(p, pre + "cond_to_qkv", modulate(c, cs_msa, csh_msa)).view(L, 3, H, HD)
        qc, kc = _qknorm(p, pre + "cond_qk_norm.", qkvc[:, 0], qkvc[:, 1])
        if L > 5:
            qc = torch.cat([qc[:5], rope_nd(qc[5:], cpos, 64.0)])
            kc = torch.cat([kc[:5], rope_nd(kc[5:], cpos, 64.0)])
        hc = attention(qc, kc, qkvc[:, 2]).reshape(L, D)
        c = c + linear(p, pre + "cond_to_out", hc) * cg_msa
        # bidirectional cross attention (no QK-norm, no RoPE)
        q, k, v = linear(p, pre + "to_qkv_cross", modulate(x, s_cr, sh_cr)).view(N, 3, H, HD).unbind(1)
        qc, kc, vc = linear(p, pre + "cond_to_qkv_cross", modulate(c, cs_cr, csh_cr)).view(L, 3, H, HD).unbind(1)
        hx = attention(q, kc, vc).reshape(N, D)
        hcx = attention(qc, k, v).reshape(L, D)
        x = x + linear(p, pre + "to_out_cross", hx) * g_cr
        c = c + linear(p, pre + "cond_to_out_cross", hcx) * cg_cr
    else:
        cs_cr, csh_cr = gates["cond"][b]
        L = c.shape[0]
        q = linear(p, pre + "to_q_cross", modulate(x, s_cr, sh_cr)).view(N, H, HD)
        kv = linear(p, pre + "cond_to_kv_cross", modulate(c, cs_cr, csh_cr)).view(L, 2, H, HD)
        x = x + linear(p, pre + "to_out_cross", attention(q, kv[:, 0], kv[:, 1]).reshape(N, D)) * g_cr

    # FFN with depthwise conv and SwiGLU (lat_dit.py:477-484; swiglu(g, a) = silu(g) * a)
    h = linear(p, pre + "ffn0", modulate(x, s_mlp, sh_mlp))
    h = dwconv27(h, p[pre + "ffn_conv.weight"], p[pre + "ffn_conv.bias"], geom.conv_indices)
    a, g = h.chunk(2, -1)
    x = x + linear(p, pre + "ffn1", F.silu(g) * a) * g_mlp

    if b < cfg.cond_depth:
        a, g = linear(p, pre + "cond_ffn0", modulate(c, cs_mlp, csh_mlp)).chunk(2, -1)
        c = c + linear(p, pre + "cond_ffn1", F.silu(g) * a) * cg_mlp
    return x, c


def flow_forward(p: Params, cfg: ModelConfig, xt_sorted: torch.Tensor, t_val: float,
                 context: Optional[torch.Tensor], geom: Geometry) -> torch.Tensor:
    """``FlowModel.forward`` on one sample in lexicographic order -> [N,16] fp32.
    ``context`` is [L,D] (after image_map); pass zeros for the uncond branch."""
    gates = time_gates(p, cfg, t_val)
    x = F.linear(xt_sorted.float(), p["flow.patchify.weight"])
    c = context.float()
    cpos = cond_positions(c.shape[0]) if c.shape[0] > 5 else None
    for b in range(cfg.depth):
        x, c = block_forward(p, cfg, b, x, c, gates, geom, cpos)
    o_s, o_sh = gates["out"]
    return F.linear(modulate(x, o_s, o_sh), p["flow.unpatchify.weight"])


def block_forward_1tok(p: Params, cfg: ModelConfig, b: int, x: torch.Tensor, c: torch.Tensor,
                       ln_c: Optional[torch.Tensor], gates: dict, geom: Geometry):
    """One block of the exact 1-token zero-context branch (``lib/fast_flow.py:1702-1794`` for
    the context blocks, ``:2295-2309`` for the others).  ``c`` is the single context token
    [1,D]; ``ln_c`` its LayerNorm after the last context block (None until a plain block
    computes it).  Returns (x, c, ln_c)."""
    H, HD, D = cfg.heads, cfg.head_dim, cfg.dim
    N = x.shape[0]
    pre = f"flow.blocks.{b}."
    s_msa, sh_msa, g_msa, s_cr, sh_cr, g_cr, s_mlp, sh_mlp, g_mlp = gates["blocks"][b]
    qkv = linear(p, pre + "to_qkv", modulate(x, s_msa, sh_msa)).view(N, 3, H, HD)
    q, k = _qknorm(p, pre + "qk_norm.", qkv[:, 0], qkv[:, 1])
    q, k = rope_nd(q, geom.pos3, 128.0), rope_nd(k, geom.pos3, 128.0)
    fwd, bwd = geom.orders[b % len(geom.orders)]
    qs, ks, vs = q[fwd], k[fwd], qkv[:, 2][fwd]
    o = torch.empty_like(qs)
    cu = geom.cu_seqlens
    for i in range(len(cu) - 1):
        o[cu[i]:cu[i + 1]] = attention(qs[cu[i]:cu[i + 1]], ks[cu[i]:cu[i + 1]], vs[cu[i]:cu[i + 1]])
    x = x + linear(p, pre + "to_out", o[bwd].reshape(N, D)) * g_msa
    if b < cfg.cond_depth:
        cs_msa, csh_msa, cg_msa, cs_cr, csh_cr, cg_cr, cs_mlp, csh_mlp, cg_mlp = gates["cond"][b]
        vcs = linear(p, pre + "cond_to_qkv", modulate(c, cs_msa, csh_msa))[:, 2 * D:]
        c = c + linear(p, pre + "cond_to_out", vcs) * cg_msa
        qkvc = linear(p, pre + "cond_to_qkv_cross", modulate(c, cs_cr, csh_cr))
        qc, vc = qkvc[:, :D].view(1, H, HD), qkvc[:, 2 * D:]
        x_const = linear(p, pre + "to_out_cross", vc)           # attention over equal keys -> V_c
        kv = linear(p, pre + "to_qkv_cross", modulate(x, s_cr, sh_cr))[:, D:].view(N, 2, H, HD)
        hcx = attention(qc, kv[:, 0], kv[:, 1]).reshape(1, D)   # one query over N keys
        x = x + x_const * g_cr
        c = c + linear(p, pre + "cond_to_out_cross", hcx) * cg_cr
    else:
        if ln_c is None:
            ln_c = layer_norm(c)
        cs_cr, csh_cr = gates["cond"][b]
        vc = linear(p, pre + "cond_to_kv_cross", ln_c * (1 + cs_cr) + csh_cr)[:, D:]
        x = x + linear(p, pre + "to_out_cross", vc) * g_cr
    h = linear(p, pre + "ffn0", modulate(x, s_mlp, sh_mlp))
    h = dwconv27(h, p[pre + "ffn_conv.weight"], p[pre + "ffn_conv.bias"], geom.conv_indices)
    a, g = h.chunk(2, -1)
    x = x + linear(p, pre + "ffn1", F.silu(g) * a) * g_mlp
    if b < cfg.cond_depth:
        a, g = linear(p, pre + "cond_ffn0", modulate(c, cs_mlp, csh_mlp)).chunk(2, -1)
        c = c + linear(p, pre + "cond_ffn1", F.silu(g) * a) * cg_mlp
    return x, c, ln_c


def flow_forward_1tok(p: Params, cfg: ModelConfig, xt_sorted: torch.Tensor, t_val: float,
                      geom: Geometry) -> torch.Tensor:
    """Exact 1-token restatement of the zero-context branch (``lib/fast_flow.py``
    ``:937-958, 1702-1794, 2295-2309``).  With an all-zero context every
    context token stays identical, so self-attention returns V, x->context
    attention returns V_c, and context->x is a single query over N keys."""
    gates = time_gates(p, cfg, t_val)
    x = F.linear(xt_sorted.float(), p["flow.patchify.weight"])
    c = torch.zeros(1, cfg.dim)
    ln_c = None
    for b in range(cfg.depth):
        x, c, ln_c = block_forward_1tok(p, cfg, b, x, c, ln_c, gates, geom)
    o_s, o_sh = gates["out"]
    return F.linear(modulate(x, o_s, o_sh), p["flow.unpatchify.weight"])


# ----------------------------------------------------------------------------- sampler

def build_schedule(num_steps: int = 4, n_guided: int = 3, rescale_t: float = 3.0,
                   cfg_range=(0.5, 1.0)):
    """Piecewise schedule of ``lib/fast_sampler.py:698-725`` (qaoa disabled):
    u runs 1 -> u_low over the guided steps and u_low -> 0 over the rest,
    t = r*u / (1 + (r-1)*u).  For 4 steps, r=3: t = [1, .9, .75, .5, 0]."""
    t_low = float(cfg_range[0])
    u_low = t_low / (rescale_t - (rescale_t - 1.0) * t_low)
    n_unguided = num_steps - n_guided
    ug = torch.linspace(1.0, u_low, n_guided + 1, dtype=torch.float32)
    uu = torch.linspace(u_low, 0.0, n_unguided + 1, dtype=torch.float32)
    u = torch.cat([ug[:-1], uu])
    t = rescale_t * u / (1.0 + (rescale_t - 1.0) * u)
    return t, [True] * n_guided + [False] * n_unguided


def cfg_reuse_delta(v_pos: torch.Tensor, last_neg: torch.Tensor, xt: torch.Tensor,
                    last_neg_x0: Optional[torch.Tensor], t_eval: float, zero_star: bool = True,
                    endpoint_blend: float = 0.08, hf_boost: float = 0.035, freq_decoupled: bool = True) -> torch.Tensor:
    """The CFG delta of a guided step that reuses the last unconditional velocity
    (``cfg_cache_mode`` "neg_reuse", ``lib/fast_flow.py:2844-2873``, non-QAOA branch): the
    candidate is ``last_neg`` blended toward its clean endpoint while t > 0.25, projected with
    CFG-Zero*'s clamped scale, then its per-channel row mean is used for the high-frequency boost."""
    if not zero_star:
        return v_pos - last_neg
    cand = last_neg
    if endpoint_blend > 0.0 and last_neg_x0 is not None and t_eval > 0.25:
        cand = (1.0 - endpoint_blend) * last_neg + endpoint_blend * ((xt - last_neg_x0) * (1.0 / t_eval))
    s = ((v_pos * cand).sum() / (cand * cand).sum().clamp_min(1e-6)).clamp(0.90, 1.10)
    delta = v_pos - s * cand
    if freq_decoupled and hf_boost > 0.0 and v_pos.shape[0] > 1:
        dc = delta.mean(dim=0, keepdim=True)
        delta = delta + hf_boost * max(0.0, 1.0 - t_eval) * (delta - dc)
    return delta


def should_eval_uncond(step: int, n_guided: int, cfg_stride: int, eval_uncond_steps) -> bool:
    """``lib/fast_sampler.py:754-768`` for the "neg_reuse" mode."""
    if eval_uncond_steps:
        return step in eval_uncond_steps
    if cfg_stride <= 1:
        return True
    if step == 0 or step == n_guided - 1:
        return True
    return step % cfg_stride == 0


def sample(p: Params, cfg: ModelConfig, vox: np.ndarray, context: torch.Tensor, noise: torch.Tensor,
           guidance_scale: float = 3.0, num_steps: int = 4, n_guided: int = 3,
           rescale_t: float = 3.0, cfg_range=(0.5, 1.0), one_token_uncond: bool = True,
           cfg_reuse: Optional[dict] = None):
    """Exact Euler + CFG sampler (``core.py:148-177`` update rule, fast-path
    schedule and unpermute/denormalize ``lib/fast_flow.py:2568-2576,
    2836, 3288, 3306-3313``).  ``noise`` is [N,16] in the caller's voxel
    order; returns [N,16] latents in that order.  ``cfg_reuse`` (a dict with
    ``eval_uncond_steps``, ``cfg_stride`` and the ``cfg_reuse_delta`` options) switches on the
    approximate CFG cache: guided steps it skips reuse the last unconditional velocity
    (``lib/fast_flow.py:2791-2887``)."""
    geom = build_geometry(vox, cfg)
    xt = noise.float()[geom.perm]
    t_seq, guided = build_schedule(num_steps, n_guided, rescale_t, cfg_range)
    tl = t_seq.tolist()
    last_neg = last_x0 = None
    opts = dict(cfg_reuse or {})
    steps, stride = opts.pop("eval_uncond_steps", [0, 2]), opts.pop("cfg_stride", 2)
    for i in range(num_steps):
        v = flow_forward(p, cfg, xt, tl[i], context, geom)
        if guided[i] and guidance_scale > 0:
            if cfg_reuse is None or last_neg is None or should_eval_uncond(i, n_guided, stride, steps):
                if one_token_uncond:
                    vn = flow_forward_1tok(p, cfg, xt, tl[i], geom)
                else:
                    vn = flow_forward(p, cfg, xt, tl[i], torch.zeros_like(context), geom)
                if cfg_reuse is not None:
                    last_neg, last_x0 = vn, xt - tl[i] * vn
                v = v + guidance_scale * (v - vn)
            else:
                v = v + guidance_scale * cfg_reuse_delta(v, last_neg, xt, last_x0, tl[i], **opts)
        xt = xt - (tl[i] - tl[i + 1]) * v
    out = xt[geom.up_widx]
    return (out * p["std"] + p["mean"]) * cfg.latent_scale
