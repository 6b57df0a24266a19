"""``OptimizedLatDitRunner``: the lat_dit forward pass on the sm_100a kernels.

Call surface of the reference's ``lib/fast_flow.py`` (``__init__``,
``_prepare_weights_and_buffers`` ``:134-354``, ``_get_time_gates`` ``:455-654``,
``_prepare_sample_geometry`` ``:657-783``, ``forward_flow_fast`` ``:786-2497``,
``warmup`` ``:2500-2520``, ``sample_fast`` ``:2523-3313``), exact path only.

Per NFE the voxel stream x [N, D] (bf16, lexicographic voxel order) goes
through 24 blocks.  Linears run on this package's tcgen05 GEMM (bf16 in, fp32
accumulate in TMEM) and, for the one-row context vector of the 1-token branch
and the time gates, on its GEMV kernel; everything between them is fused
gate-add + LayerNorm + AdaLN, QK-RMSNorm + 3D RoPE + Hilbert gather,
tcgen05 flash attention with the window un-permutation fused into its
epilogue, depthwise 27-tap conv with the SwiGLU fused in, output
modulation + unpatchify.  The unconditional branch is the exact 1-token
condensation: the context stream is one vector, its self- and x->context
attention collapse to linear maps and context->x is one query per head
over the N voxels.
"""
from __future__ import annotations

import math
from collections import OrderedDict
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Dict, List, Optional

import torch

from . import fast_kernels as fk
from .fast_sampler import SolverConfig, build_schedule, should_eval_uncond
from .model import LatDitArch, LatDitModel
from .runtime import FlowMatchSamplingParams, LatDitConditioning

BF16 = torch.bfloat16
F32 = torch.float32

# Kernel classes of the forward (the kernel timer's keys) and what bounds each: "tensor"
# classes count FLOPs, "hbm" classes count algorithmic bytes (each tensor read or written once).
KERNEL_CLASSES = {
    "attention_window_self": "tensor", "attention_voxel_to_context": "tensor",
    "attention_context_to_voxel": "tensor", "attention_context_self": "tensor",
    "gemm_qkv_fused": "tensor", "gemm_voxel": "tensor", "gemm_context": "tensor",
    "dwconv27_swiglu": "hbm", "gate_add_modulate": "hbm", "single_query_context_to_voxel": "hbm",
    "unpatchify_project": "hbm",
}


def _time_encoding(t: torch.Tensor, dim: int, max_period: float = 10000.0) -> torch.Tensor:
    """[cos(t w), sin(t w)], w = exp(-ln(1e4) 2i/dim), fp64 (``BK/base_models/fourier_utils.py:33-44``)."""
    omega = torch.exp(-math.log(max_period) * torch.arange(0, dim, 2, dtype=torch.float64, device=t.device) / dim)
    f = t.to(torch.float64)[..., None] * omega
    return torch.cat([torch.cos(f), torch.sin(f)], -1).float()


@dataclass
class _SampleGraph:
    """A captured sample: the graph and the buffers it reads and writes."""
    graph: "torch.cuda.CUDAGraph"
    geom: Dict[str, Any]
    context: torch.Tensor
    noise: torch.Tensor
    out: torch.Tensor


def _copy_into(dst, src) -> None:
    """Copy every tensor of a geometry dict (nested lists/tuples) into its counterpart."""
    if torch.is_tensor(dst):
        if dst is not src:
            dst.copy_(src)
    elif isinstance(dst, dict):
        for k, v in dst.items():
            _copy_into(v, src[k])
    elif isinstance(dst, (list, tuple)):
        for a, b in zip(dst, src):
            _copy_into(a, b)


class OptimizedLatDitRunner:
    """Runs ``FlowModel`` NFEs and the exact sampler on one CUDA device."""

    def __init__(self, model, solver_config: Optional[SolverConfig] = None, weights_dir: Optional[Path] = None,
                 device: Optional[torch.device] = None, cuda_graph: bool = False):
        if hasattr(model, "core") and not isinstance(model, LatDitModel):   # a reference LatDitModel
            core = model.core
            mc = dict(core.model_config, latent_scale=float(core.latent_scale))
            model = LatDitModel.from_state_dict(core.state_dict(), mc)
        self.model: LatDitModel = model
        self.arch: LatDitArch = model.arch
        self.solver_config = solver_config or SolverConfig()
        self.weights_dir = weights_dir
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if self.device.type != "cuda":
            raise RuntimeError("OptimizedLatDitRunner runs on CUDA only")
        a = self.arch
        self.dim, self.head_dim, self.num_heads = a.dim, a.head_dim, a.heads
        self.depth, self.cond_depth, self.res = a.depth, a.cond_depth, a.res
        self.latent_dim, self.latent_scale = a.latent_dim, a.latent_scale
        self._time_gates_cache: Dict[float, Dict[str, torch.Tensor]] = {}
        self._rope_2d_cache: Dict[int, tuple] = {}
        self._b0_share = None
        # when a dict, every launch of the forward's main kernels appends (start event, end
        # event, algorithmic units, whether another NFE shared the GPU) under its kernel
        # class (KERNEL_CLASSES): the benchmark's in-step measurement of each kernel
        self.kernel_timer: Optional[Dict[str, list]] = None
        # when a set, only these kernel classes are timed (the others launch without events)
        self.kernel_timer_kinds: Optional[set] = None
        self._nfe_shared = False
        self._ctx_rows = -1            # rows of the context stream in the current NFE (GEMM classes)
        # the context stream of the context blocks runs on its own CUDA stream
        self.overlap_context = True
        self._ctx_streams: Dict[int, torch.cuda.Stream] = {}
        # the 1-token NFE of a guided step runs on its own stream beside the conditional one
        self.overlap_branches = True
        self._neg_stream: Optional[torch.cuda.Stream] = None
        # the self-attention to_qkv GEMM runs QK-norm, RoPE3D and the window-order scatter
        # in its epilogue (tcgen05 GEMM) where the head layout allows (head_dim 96 or 128,
        # an even number of heads: a pair tile holds two whole heads of one section)
        self.fused_qkv = self.head_dim in (96, 128) and self.num_heads % 2 == 0
        # the 1-token branch's single query over the voxel rows without forming K/V takes up to
        # 16 heads and a width that is a multiple of 128 (at most 2048); other widths form K/V
        self._wide_1q = self.num_heads <= 16 and self.dim % 128 == 0 and self.dim <= 2048 and self.head_dim <= 256
        # CUDA-graph replay of the sampler (per voxel count, context length and schedule)
        self.cuda_graph = bool(cuda_graph)
        self._graphs: "OrderedDict[tuple, _SampleGraph]" = OrderedDict()
        self.max_graphs = 4
        self._prepare_weights_and_buffers()

    # ------------------------------------------------------------------ weights
    def _prepare_weights_and_buffers(self) -> None:
        """bf16 device copies of the linears, fp32 conv / unpatchify / gate weights,
        the 1-token collapsed maps, RoPE tables and the schedule's gate vectors."""
        sd, a, dev = self.model.state, self.arch, self.device
        D = a.dim

        def bf(k):
            return sd[k].to(dev, BF16).contiguous()

        def f32(k):
            return sd[k].to(dev, F32).contiguous()

        self.W_patch = f32("flow.patchify.weight")                 # [D, 16]
        self.W_unpatch = f32("flow.unpatchify.weight")             # [16, D]
        self.W_unpatch3 = fk.split_weight3(self.W_unpatch)         # [48, D] bf16 hi / mid / lo parts
        self.W_image = bf("image_map.weight")
        self.b_image = bf("image_map.bias")
        self.W_t0, self.b_t0 = f32("flow.time_embed.0.weight"), f32("flow.time_embed.0.bias")
        self.W_t2, self.b_t2 = f32("flow.time_embed.2.weight"), f32("flow.time_embed.2.bias")
        self.W_og, self.b_og = f32("flow.out_gates.weight"), f32("flow.out_gates.bias")
        cd = a.cond_depth
        self.W_g = torch.cat([f32(f"flow.blocks.{b}.gates.weight") for b in range(a.depth)])
        self.b_g = torch.cat([f32(f"flow.blocks.{b}.gates.bias") for b in range(a.depth)])
        self.W_cg9 = torch.cat([f32(f"flow.blocks.{b}.cond_gates.weight") for b in range(cd)]) if cd else None
        self.b_cg9 = torch.cat([f32(f"flow.blocks.{b}.cond_gates.bias") for b in range(cd)]) if cd else None
        nc = range(cd, a.depth)
        self.W_cg2 = torch.cat([f32(f"flow.blocks.{b}.cond_gates.weight") for b in nc]) if a.depth > cd else None
        self.b_cg2 = torch.cat([f32(f"flow.blocks.{b}.cond_gates.bias") for b in nc]) if a.depth > cd else None

        Fh = a.ffn_dim
        self.ffn_interleaved = (2 * Fh) % 128 == 0
        self.ffn_perm = torch.arange(2 * Fh, device=self.device).view(2, Fh // 2, 2).permute(1, 0, 2).reshape(-1)
        self.blocks: List[Dict[str, torch.Tensor]] = []
        # per block: the conv weights hold bf16 values (a bf16 model upcast), so the conv may
        # take its bf16-operand FMAs, which give the same bits
        self.conv_bf16w: List[bool] = []
        for b in range(a.depth):
            p = f"flow.blocks.{b}."
            w = {n: bf(p + n + ".weight") for n in ("to_qkv", "to_out", "to_out_cross", "ffn0", "ffn1")}
            w.update({n + "_b": bf(p + n + ".bias") for n in ("to_qkv", "to_out", "to_out_cross", "ffn0", "ffn1")})
            w["conv_w"] = f32(p + "ffn_conv.weight").reshape(27, -1).contiguous()
            w["conv_b"] = f32(p + "ffn_conv.bias")
            if self.ffn_interleaved:
                # hidden columns (a[2k], a[2k+1], gate[2k], gate[2k+1]): the layout the staged
                # conv reads; only the order of ffn0's outputs changes
                w["ffn0"] = w["ffn0"][self.ffn_perm].contiguous()
                w["ffn0_b"] = w["ffn0_b"][self.ffn_perm].contiguous()
                w["conv_w"] = w["conv_w"][:, self.ffn_perm].contiguous()
                w["conv_b"] = w["conv_b"][self.ffn_perm].contiguous()
            self.conv_bf16w.append(fk.weights_are_bf16(w["conv_w"]))
            w["qs"], w["ks"] = f32(p + "qk_norm.q_scale"), f32(p + "qk_norm.k_scale")
            if b < cd:
                for n in ("cond_to_qkv", "cond_to_out", "to_qkv_cross", "cond_to_qkv_cross", "cond_to_out_cross",
                          "cond_ffn0", "cond_ffn1"):
                    w[n], w[n + "_b"] = bf(p + n + ".weight"), bf(p + n + ".bias")
                w["cqs"], w["cks"] = f32(p + "cond_qk_norm.q_scale"), f32(p + "cond_qk_norm.k_scale")
                # 1-token maps (lib/fast_flow.py:195-309), collapsed in fp32 then rounded
                Wv = f32(p + "cond_to_qkv.weight")[2 * D:]
                bv = f32(p + "cond_to_qkv.bias")[2 * D:]
                Wo, bo = f32(p + "cond_to_out.weight"), f32(p + "cond_to_out.bias")
                w["msa1_w"], w["msa1_b"] = (Wo @ Wv).to(BF16), (Wo @ bv + bo).to(BF16)
                Wqx = f32(p + "cond_to_qkv_cross.weight")
                bqx = f32(p + "cond_to_qkv_cross.bias")
                Wox, box = f32(p + "to_out_cross.weight"), f32(p + "to_out_cross.bias")
                w["qcr1_w"] = torch.cat([Wqx[:D], Wox @ Wqx[2 * D:]]).to(BF16).contiguous()
                w["qcr1_b"] = torch.cat([bqx[:D], Wox @ bqx[2 * D:] + box]).to(BF16).contiguous()
                w["kvx_w"] = w["to_qkv_cross"][D:].contiguous()          # K,V rows of to_qkv_cross
                w["kvx_b"] = w["to_qkv_cross_b"][D:].contiguous()
            else:
                for n in ("to_q_cross", "cond_to_kv_cross"):
                    w[n], w[n + "_b"] = bf(p + n + ".weight"), bf(p + n + ".bias")
                Wv = f32(p + "cond_to_kv_cross.weight")[D:]
                bv = f32(p + "cond_to_kv_cross.bias")[D:]
                Wox, box = f32(p + "to_out_cross.weight"), f32(p + "to_out_cross.bias")
                w["cr1_w"], w["cr1_b"] = (Wox @ Wv).to(BF16), (Wox @ bv + box).to(BF16)
            self.blocks.append(w)
        if a.depth > cd:
            # the constant cross-attention maps of the plain blocks, one batched GEMV per NFE
            self.cr1_w_all = torch.stack([self.blocks[b]["cr1_w"] for b in range(cd, a.depth)]).contiguous()
            self.cr1_b_all = torch.stack([self.blocks[b]["cr1_b"] for b in range(cd, a.depth)]).contiguous()
        self.mean = f32("mean").reshape(1, -1)
        self.std = f32("std").reshape(1, -1)
        self._denorm_scale = (self.std * a.latent_scale).reshape(-1).contiguous()
        self._denorm_shift = (self.mean * a.latent_scale).reshape(-1).contiguous()
        self.cos3, self.sin3 = fk.precompute_rope_3d_table(a.res, 128.0, a.head_dim, device=dev)
        self._time_gates_cache.clear()
        if self.solver_config.precompute_time_gates:
            t_seq, _, _ = build_schedule(self.solver_config)
            for t in t_seq.tolist()[:-1]:
                self._get_time_gates(float(t))

    def _run(self, kind: str, units: float, fn, *args, **kw):
        """fn(*args, **kw); with the kernel timer on, CUDA events around it on the current
        stream, filed under ``kind`` with its algorithmic units (FLOPs or bytes)."""
        kt = self.kernel_timer
        if kt is None or (self.kernel_timer_kinds is not None and kind not in self.kernel_timer_kinds):
            return fn(*args, **kw)
        e0 = torch.cuda.Event(enable_timing=True)
        e0.record()
        out = fn(*args, **kw)
        e1 = torch.cuda.Event(enable_timing=True)
        e1.record()
        kt.setdefault(kind, []).append((e0, e1, float(units), self._nfe_shared))
        return out

    def _lin(self, a: torch.Tensor, w: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
        """A block linear on the tcgen05 GEMM (voxel rows or context rows)."""
        kind = "gemm_context" if a.shape[0] == self._ctx_rows else "gemm_voxel"
        return self._run(kind, 2.0 * a.shape[0] * a.shape[1] * w.shape[0], fk.linear, a, w, b)

    def _att(self, kind: str, q, k, v, cu_q, cu_k, **kw) -> torch.Tensor:
        """Attention launch; FLOPs 4 * sum over segments of n_q * n_k * D."""
        units = 0.0
        if self.kernel_timer is not None:
            units = 4.0 * self.dim * sum((cu_q[i + 1] - cu_q[i]) * (cu_k[i + 1] - cu_k[i]) for i in range(len(cu_q) - 1))
        return self._run(kind, units, fk.attention, q, k, v, cu_q, cu_k, self.num_heads, self.head_dim, **kw)

    def _gate_add_mod(self, x, h, g, s1, sh, broadcast_h: bool = False) -> torch.Tensor:
        """x += g * h; returns LN(x) * s1 + sh (bytes: x read and written, h read, h_mod written)."""
        nb = x.shape[0] * x.shape[1] * 2.0 * (3 if broadcast_h else 4)
        return self._run("gate_add_modulate", nb, fk.fast_gate_add_and_modulate, x, h, g, s1, sh,
                         broadcast_h=broadcast_h)

    def _unpatchify(self, y: torch.Tensor) -> torch.Tensor:
        """[N,16] fp32 velocity from the output-modulated rows y = bf16(LN(x) * s1 + sh): the
        projection of ``lib/fast_kernels.py:613-648`` with its fp32 weight (bytes: y read, out written)."""
        return self._run("unpatchify_project", y.shape[0] * (y.shape[1] * 2.0 + 64.0), fk.unpatchify_project, y,
                         self.W_unpatch3)

    def _get_rope_2d_table(self, cond_size: int):
        if cond_size not in self._rope_2d_cache:
            self._rope_2d_cache[cond_size] = fk.precompute_rope_2d_cond(cond_size, 64.0, self.head_dim,
                                                                         device=self.device)
        return self._rope_2d_cache[cond_size]

    @torch.no_grad()
    def _get_time_gates(self, t_val: float, device=None, dtype=None, clf_token=None) -> Dict[str, torch.Tensor]:
        """fp32 gate vectors at time t (``lat_dit.py:747-750, 391-392, 409-410, 463-464, 817``).
        Rows 0/3/6 of the 9-gate blocks hold 1 + scale."""
        key = round(float(t_val), 7)
        hit = self._time_gates_cache.get(key)
        if hit is not None:
            return hit
        a, D = self.arch, self.dim
        t = torch.full((1,), float(t_val) * 1000.0, dtype=F32, device=self.device)
        enc = _time_encoding(t, a.time_pos_features)[0].contiguous()
        h = fk.gemv(enc, self.W_t0, self.b_t0, out_dtype=F32, silu_out=True)
        clf = fk.gemv(h, self.W_t2, self.b_t2, out_dtype=F32, silu_out=True)
        g = fk.gemv(clf, self.W_g, self.b_g, out_dtype=F32).view(a.depth, 9, D).clone()
        g[:, 0::3] += 1.0
        out = {"clf": clf, "blk": g.contiguous()}
        if self.W_cg9 is not None:
            c9 = fk.gemv(clf, self.W_cg9, self.b_cg9, out_dtype=F32).view(a.cond_depth, 9, D).clone()
            c9[:, 0::3] += 1.0
            out["cond9"] = c9.contiguous()
        if self.W_cg2 is not None:
            c2 = fk.gemv(clf, self.W_cg2, self.b_cg2, out_dtype=F32).view(a.depth - a.cond_depth, 2, D).clone()
            c2[:, 0] += 1.0
            out["cond2"] = c2.contiguous()
        o = fk.gemv(clf, self.W_og, self.b_og, out_dtype=F32).view(2, D).clone()
        o[0] += 1.0
        out["out"] = o.contiguous()
        self._time_gates_cache[key] = out
        return out

    # ------------------------------------------------------------------ geometry
    @torch.no_grad()
    def _prepare_sample_geometry(self, vox_idxs: List[torch.Tensor], context: torch.Tensor) -> Dict[str, Any]:
        """Static geometry of one sample, computed once per sample on the GPU."""
        if len(vox_idxs) != 1:
            raise NotImplementedError("batch_size 1 per runner call (samples shard across calls / GPUs)")
        vox = vox_idxs[0].to(self.device, torch.int32).contiguous()
        N = vox.shape[0]
        perm, up_widx, h_coords = fk.lex_perm(vox)
        order_caches = fk.build_order_caches_fast(h_coords, [N], self.arch.orders,
                                                  {"patch_size": self.arch.patch_size}, coord_bound=1024)
        conv_indices = fk.build_conv_indices_fast(h_coords, already_sorted=True)
        # staging plan of the fused conv + SwiGLU: blocks of rows along the first Hilbert order
        conv_plan = fk.build_conv_plan(conv_indices, order_caches[0][0]) if self.ffn_interleaved else None
        L = context.shape[-2]
        cond_size = int(round(math.sqrt(max(L - 5, 0))))
        if L > 5 and cond_size * cond_size != L - 5:
            raise ValueError(f"context of {L} tokens: expected 5 prefix tokens and a square grid of image tokens")
        cos2, sin2 = self._get_rope_2d_table(cond_size) if L > 5 else (None, None)
        return {"N": N, "batch_size": 1, "sizes": [N], "layout": [slice(0, N)], "perm": perm, "up_widx": up_widx,
                "h_coords": h_coords, "cos_vox": self.cos3, "sin_vox": self.sin3, "cos_cond_2d": cos2,
                "sin_cond_2d": sin2, "order_caches": order_caches, "conv_indices": conv_indices,
                "conv_plan": conv_plan,
                "q_seqlens": [0, N], "q_maxlen": N, "kv_seqlens_full": [0, L], "kv_maxlen_full": L,
                "kv_seqlens_1tok": [0, 1], "kv_maxlen_1tok": 1}

    # ------------------------------------------------------------------ forward
    def _self_attention(self, b: int, h_mod: torch.Tensor, geom) -> torch.Tensor:
        """Window self-attention in Hilbert order orders[b % 4]; returns to_out(o) [N, D]."""
        w, H, HD = self.blocks[b], self.num_heads, self.head_dim
        D = self.dim
        fwd, bwd, cu, _ = geom["order_caches"][b % len(geom["order_caches"])]
        if self.fused_qkv:
            qkv_s = self._run("gemm_qkv_fused", 2.0 * h_mod.shape[0] * D * 3 * D, fk.linear_qkv_rope3d, h_mod,
                              w["to_qkv"], w["to_qkv_b"], w["qs"], w["ks"], self.cos3, self.sin3, geom["h_coords"],
                              bwd, H, HD)
        else:
            qkv = self._lin(h_mod, w["to_qkv"], w["to_qkv_b"])
            qkv_s = fk.fused_qknorm_rope3d_gather(qkv, w["qs"], w["ks"], self.cos3, self.sin3, geom["h_coords"], fwd,
                                                  H, HD)
        o = self._att("attention_window_self", qkv_s[:, :D], qkv_s[:, D:2 * D], qkv_s[:, 2 * D:], cu.host, cu.host,
                      out_rows=fwd)
        return self._lin(o, w["to_out"], w["to_out_b"])

    def _ffn(self, b: int, h_mod: torch.Tensor, geom) -> torch.Tensor:
        w = self.blocks[b]
        h2 = self._lin(h_mod, w["ffn0"], w["ffn0_b"])
        n, f2 = h2.shape
        conv_bytes = n * f2 * 2.0 + n * (f2 // 2) * 2.0 + 27 * f2 * 4.0 + n * 27 * 4.0
        if self.ffn_interleaved:
            y = self._run("dwconv27_swiglu", conv_bytes, fk.fast_sparse_conv3d_swiglu_planned, h2, w["conv_w"],
                          w["conv_b"], geom["conv_plan"], bf16_weights=self.conv_bf16w[b])
        else:
            y = self._run("dwconv27_swiglu", conv_bytes, fk.fast_sparse_conv3d, h2, w["conv_w"], w["conv_b"],
                          geom["conv_indices"], fuse_swiglu=True)
        return self._lin(y, w["ffn1"], w["ffn1_b"])

    @torch.no_grad()
    def forward_flow_fast(self, xt_sorted: torch.Tensor, t_val: float, context: torch.Tensor,
                          clf_token: Optional[torch.Tensor], geom: Dict[str, Any], *, uncond: bool = False,
                          **unused) -> torch.Tensor:
        """One NFE on ``xt_sorted`` [N,16] fp32 (lexicographic order) -> velocity [N,16] fp32.
        ``context`` is the image context after ``image_map`` ([1,L,D] or [L,D]); ignored when
        ``uncond`` (exact 1-token branch)."""
        if uncond and self.solver_config.uncond_1token_condensation:
            return self._forward_uncond_1tok(xt_sorted, t_val, geom)
        tg = self._get_time_gates(t_val)
        G, CG9, CG2, OG = tg["blk"], tg.get("cond9"), tg.get("cond2"), tg["out"]
        H, HD, D, cd = self.num_heads, self.head_dim, self.dim, self.cond_depth
        N = xt_sorted.shape[0]
        c = (torch.zeros_like(context) if uncond else context).reshape(-1, D).to(BF16).contiguous().clone()
        L = c.shape[0]
        self._ctx_rows = L if L != N else -1
        cos2, sin2 = geom["cos_cond_2d"], geom["sin_cond_2d"]
        x = fk.patchify(xt_sorted, self.W_patch)
        h_mod = fk.fast_modulate(x, None, G[0, 0], G[0, 1])
        c_mod = fk.fast_modulate(c, None, CG9[0, 0], CG9[0, 1]) if cd > 0 else None
        share = self.solver_config.ditfastattn_b0_msa_share
        # The context stream of the context blocks runs on a second CUDA stream: it meets the
        # voxel stream only at the cross-attention (q/k/v of both sides) and after the last
        # context block (the frozen context feeds the remaining blocks).  Tensors that cross
        # streams are recorded on the stream that reads them.
        main = torch.cuda.current_stream(self.device)
        side = self._context_stream() if (cd > 0 and self.overlap_context) else main
        if side is not main:
            side.wait_stream(main)
            c.record_stream(side)
            c_mod.record_stream(side)
        for b in range(self.depth):
            w = self.blocks[b]
            if b < cd:
                CG = CG9[b]
                with torch.cuda.stream(side):
                    qkvc = self._lin(c_mod, w["cond_to_qkv"], w["cond_to_qkv_b"])
                    fk.fused_qknorm_rope2d_cond_inplace(qkvc, w["cqs"], w["cks"], cos2, sin2, H, HD, n_prefix=5)
                    oc = self._att("attention_context_self", qkvc[:, :D], qkvc[:, D:2 * D], qkvc[:, 2 * D:],
                                   [0, L], [0, L])
                    hc = self._lin(oc, w["cond_to_out"], w["cond_to_out_b"])
                    c_mod = self._gate_add_mod(c, hc, CG[2], CG[3], CG[4])
                    qkvcc = self._lin(c_mod, w["cond_to_qkv_cross"], w["cond_to_qkv_cross_b"])
            h = self._self_attention(b, h_mod, geom)
            h_mod = self._gate_add_mod(x, h, G[b, 2], G[b, 3], G[b, 4])
            if b == 0 and share:
                x0 = x.clone()
                ev0 = torch.cuda.Event()
                ev0.record()
                self._b0_share = (round(float(t_val), 7), x0, ev0)
            if b < cd:
                qkvx = self._lin(h_mod, w["to_qkv_cross"], w["to_qkv_cross_b"])
                if side is not main:
                    main.wait_stream(side)                 # qkvcc is ready
                    qkvcc.record_stream(main)
                    side.wait_stream(main)                 # qkvx is ready
                    qkvx.record_stream(side)
                with torch.cuda.stream(side):
                    ocx = self._att("attention_context_to_voxel", qkvcc[:, :D], qkvx[:, D:2 * D], qkvx[:, 2 * D:],
                                    [0, L], [0, N])
                    hcx = self._lin(ocx, w["cond_to_out_cross"], w["cond_to_out_cross_b"])
                    c_mod = self._gate_add_mod(c, hcx, CG[5], CG[6], CG[7])
                    hc2 = self._lin(c_mod, w["cond_ffn0"], w["cond_ffn0_b"])
                    hcf = self._lin(fk.fast_swiglu_from_packed(hc2), w["cond_ffn1"], w["cond_ffn1_b"])
                    if b + 1 < cd:
                        c_mod = self._gate_add_mod(c, hcf, CG[8], CG9[b + 1, 0], CG9[b + 1, 1])
                    else:
                        fk.fast_gate_add(c, hcf, CG[8])
                    if b + 1 == cd:
                        # the context is frozen from here on: the K/V of every remaining block
                        kv_frozen = self._frozen_context_kv(c, CG2)
                ox = self._att("attention_voxel_to_context", qkvx[:, :D], qkvcc[:, D:2 * D], qkvcc[:, 2 * D:], [0, N],
                               [0, L])
                hx = self._lin(ox, w["to_out_cross"], w["to_out_cross_b"])
                h_mod = self._gate_add_mod(x, hx, G[b, 5], G[b, 6], G[b, 7])
            else:
                if cd == 0 and b == 0:
                    kv_frozen = self._frozen_context_kv(c, CG2)
                q = self._lin(h_mod, w["to_q_cross"], w["to_q_cross_b"])
                kv, ready = kv_frozen[b - cd]
                if side is not main:
                    main.wait_event(ready)
                    kv.record_stream(main)
                ox = self._att("attention_voxel_to_context", q, kv[:, :D], kv[:, D:], [0, N], [0, L])
                hx = self._lin(ox, w["to_out_cross"], w["to_out_cross_b"])
                h_mod = self._gate_add_mod(x, hx, G[b, 5], G[b, 6], G[b, 7])
            hf = self._ffn(b, h_mod, geom)
            # after the last block the gate-add modulates with the output norm's scale and shift
            nxt = (G[b + 1, 0], G[b + 1, 1]) if b + 1 < self.depth else (OG[0], OG[1])
            h_mod = self._gate_add_mod(x, hf, G[b, 8], *nxt)
        if side is not main:
            main.wait_stream(side)
        return self._unpatchify(h_mod)

    def _frozen_context_kv(self, c: torch.Tensor, CG2) -> list:
        """K/V of the frozen context for every block after the context blocks, queued on the
        current stream (the context stream); each comes with an event the voxel stream waits on."""
        out = []
        for b in range(self.cond_depth, self.depth):
            C2 = CG2[b - self.cond_depth]
            w = self.blocks[b]
            cm = fk.fast_modulate(c, None, C2[0], C2[1])
            kv = self._lin(cm, w["cond_to_kv_cross"], w["cond_to_kv_cross_b"])
            ev = torch.cuda.Event()
            ev.record()
            out.append((kv, ev))
        return out

    def _context_stream(self) -> torch.cuda.Stream:
        """The context stream paired with the current stream (each NFE stream has its own)."""
        key = torch.cuda.current_stream(self.device).cuda_stream
        st = self._ctx_streams.get(key)
        if st is None:
            st = self._ctx_streams[key] = torch.cuda.Stream(self.device)
        return st

    def _forward_uncond_1tok(self, xt_sorted: torch.Tensor, t_val: float, geom) -> torch.Tensor:
        """Exact zero-context branch with a 1-token context stream (fp32 vector)."""
        tg = self._get_time_gates(t_val)
        G, CG9, CG2, OG = tg["blk"], tg.get("cond9"), tg.get("cond2"), tg["out"]
        H, HD, D, cd = self.num_heads, self.head_dim, self.dim, self.cond_depth
        key = round(float(t_val), 7)
        share = self._b0_share if (self.solver_config.ditfastattn_b0_msa_share and self._b0_share is not None
                                   and self._b0_share[0] == key
                                   and self._b0_share[1].shape[0] == xt_sorted.shape[0]) else None
        c = torch.zeros(D, dtype=F32, device=xt_sorted.device)
        # The context vector's chain (modulated GEMVs, the single query over the voxels, the
        # context FFN) runs on the context stream; it meets the voxel stream at the constant
        # cross-attention output (needed by the voxel gate-add) and at the voxel K/V (read by
        # the single-query attention).  Tensors that cross streams are recorded on the reader.
        main = torch.cuda.current_stream(self.device)
        side = self._context_stream() if self.overlap_context else main
        two = side is not main
        if two:
            side.wait_stream(main)
            c.record_stream(side)

        def mod_lin(scale1, shift, wk, bk, blk):
            """bf16 Linear(LN(c) * scale1 + shift) of the context vector (one GEMV launch)."""
            return fk.gemv(c, blk[wk], blk[bk], x_mode=fk.GEMV_X_LN_MOD, mod_scale=scale1, mod_shift=shift)

        def on_side_event():
            ev = torch.cuda.Event()
            ev.record()
            return ev

        if share is not None:
            cur = torch.cuda.current_stream(self.device)
            cur.wait_event(share[2])                  # block 0 of the conditional NFE is done
            share[1].record_stream(cur)
            x = share[1].clone()
            h_mod = fk.fast_modulate(x, None, G[0, 3], G[0, 4])
            start = 1
        else:
            x = fk.patchify(xt_sorted, self.W_patch)
            h_mod = fk.fast_modulate(x, None, G[0, 0], G[0, 1])
            start = 0
        consts = []
        for b in range(self.depth):
            w = self.blocks[b]
            if b < cd:
                CG = CG9[b]
                with torch.cuda.stream(side):
                    fk.vec_gate_residual_(c, mod_lin(CG[0], CG[1], "msa1_w", "msa1_b", w), CG[2])
                    qo = mod_lin(CG[3], CG[4], "qcr1_w", "qcr1_b", w)              # bf16 [2D]
                    q_cc, x_const = qo[:D], qo[D:]
                    q_ready = on_side_event()
            elif b == cd:
                # the context vector is frozen from here on: the constant cross-attention output
                # of every remaining block, one event each
                with torch.cuda.stream(side):
                    # one batched GEMV: block bb's map of LN(c) * (1 + cs_bb) + csh_bb
                    xc_all = fk.gemv(c, self.cr1_w_all, self.cr1_b_all, x_mode=fk.GEMV_X_LN_MOD,
                                     mod_scale=CG2[:, 0], mod_shift=CG2[:, 1])
                    ev = on_side_event()
                    consts = [(xc_all[i], ev) for i in range(self.depth - cd)]
            h = self._self_attention(b, h_mod, geom) if b >= start else None
            if h is not None and b < cd:
                h_mod = self._gate_add_mod(x, h, G[b, 2], G[b, 3], G[b, 4])
            if b < cd:
                # the context query attends over K/V = cross linear of the modulated stream;
                # attention_1q_wide reads the stream itself (K/V are never formed)
                h_kv = h_mod
                if two:
                    kv_ready = torch.cuda.Event()
                    kv_ready.record(main)
                    main.wait_event(q_ready)
                    qo.record_stream(main)
                h_mod = self._gate_add_mod(x, x_const, G[b, 5], G[b, 6], G[b, 7], broadcast_h=True)
                with torch.cuda.stream(side):
                    if two:
                        side.wait_event(kv_ready)
                        h_kv.record_stream(side)
                    if self._wide_1q:
                        o1 = self._run("single_query_context_to_voxel", h_kv.numel() * 2.0 + w["kvx_w"].numel() * 2.0,
                                       fk.attention_1q_wide, q_cc, h_kv, w["kvx_w"], w["kvx_b"], H, HD)   # bf16 [D]
                    else:
                        # widths the fused single query does not take: form K/V, then one query per head
                        kv = self._lin(h_kv, w["kvx_w"], w["kvx_b"])
                        o1 = fk.attention_1q(q_cc, kv, H, HD)
                    fk.vec_gate_residual_(c, fk.gemv(o1, w["cond_to_out_cross"], w["cond_to_out_cross_b"]), CG[5])
                    a_g = mod_lin(CG[6], CG[7], "cond_ffn0", "cond_ffn0_b", w)    # bf16 [2F]
                    # cond_ffn1(silu(g) * a): the SwiGLU of the packed vector runs in the GEMV prologue
                    fk.vec_gate_residual_(c, fk.gemv(a_g, w["cond_ffn1"], w["cond_ffn1_b"], x_mode=fk.GEMV_X_SWIGLU),
                                          CG[8])
            else:
                x_const, ready = consts[b - cd]
                if two:
                    main.wait_event(ready)
                    x_const.record_stream(main)
                if h is not None:
                    # the self-attention and the constant cross-attention gate-adds in one pass
                    # (the modulation between them feeds nothing in this branch)
                    h_mod = self._run("gate_add_modulate", x.numel() * 8.0, fk.fast_gate_add2_and_modulate, x, h,
                                      G[b, 2], x_const, G[b, 5], G[b, 6], G[b, 7])
                else:
                    h_mod = self._gate_add_mod(x, x_const, G[b, 5], G[b, 6], G[b, 7], broadcast_h=True)
            hf = self._ffn(b, h_mod, geom)
            nxt = (G[b + 1, 0], G[b + 1, 1]) if b + 1 < self.depth else (OG[0], OG[1])
            h_mod = self._gate_add_mod(x, hf, G[b, 8], *nxt)
        if two:
            main.wait_stream(side)
        return self._unpatchify(h_mod)

    # ------------------------------------------------------------------ sampler
    @torch.no_grad()
    def encode_context(self, dino_features: torch.Tensor) -> torch.Tensor:
        """image_map: [1, L, 1280] -> [L, D] bf16 (``core.py:87-97``)."""
        d = dino_features.to(self.device, BF16).reshape(-1, dino_features.shape[-1])
        return fk.linear(d, self.W_image, self.b_image)

    @torch.no_grad()
    def sample_fast(self, vox_idxs: List[torch.Tensor], conditioning: LatDitConditioning, *,
                    sampling: Optional[FlowMatchSamplingParams] = None, generator: Optional[torch.Generator] = None,
                    noise: Optional[torch.Tensor] = None) -> List[torch.Tensor]:
        """Exact Euler + CFG sampler; returns [N,16] fp32 latents in the input voxel order.
        ``noise`` ([N,16], input order) overrides the generator draw."""
        context = self.encode_context(conditioning.dino_features)
        return [self.sample_with_context(vox_idxs[0], context, sampling=sampling, generator=generator, noise=noise)]

    @torch.no_grad()
    def sample_with_context(self, vox: torch.Tensor, context: torch.Tensor, *,
                            sampling: Optional[FlowMatchSamplingParams] = None,
                            generator: Optional[torch.Generator] = None,
                            noise: Optional[torch.Tensor] = None,
                            cuda_graph: Optional[bool] = None) -> torch.Tensor:
        """The sampler on one sample with the image context already mapped ([L, D]).
        With ``cuda_graph`` (default: the runner's setting) the GPU part of the sample
        (noise gather, all NFEs, CFG + Euler, un-permutation) is captured once per
        (voxel count, context length, schedule) and replayed; the geometry is built
        eagerly for every sample and copied into the captured buffers."""
        geom = self._prepare_sample_geometry([vox], context)
        N = geom["N"]
        if noise is None:
            noise = torch.randn(N, self.latent_dim, dtype=F32, device=self.device, generator=generator)
        noise = noise.to(self.device, F32)
        tl, guided, g_scale = self._schedule(sampling)
        use_graph = self.cuda_graph if cuda_graph is None else bool(cuda_graph)
        if not use_graph:
            return self._sample_steps(geom, context, noise, tl, guided, g_scale)
        sc = self.solver_config
        key = (N, int(context.shape[-2]), tuple(tl), tuple(guided), g_scale, sc.approximate_cfg_cache,
               tuple(sc.eval_uncond_steps), sc.cfg_stride)
        entry = self._graphs.get(key)
        if entry is None:
            entry = self._capture_sample(key, geom, context, noise, tl, guided, g_scale)
        else:
            self._graphs.move_to_end(key)
            _copy_into(entry.geom, geom)
            entry.context.copy_(context)
            entry.noise.copy_(noise)
        entry.graph.replay()
        return entry.out.clone()

    def _schedule(self, sampling: Optional[FlowMatchSamplingParams]):
        """(t nodes, guided flags, guidance scale) of the solver config with the call's overrides."""
        sc = self.solver_config
        g_scale, steps_ovr, r_ovr, cr_ovr = sc.guidance_scale, None, None, None
        if sampling is not None:
            g_scale = float(sampling.guidance_scale)
            r_ovr = float(sampling.rescale_t)
            cr_ovr = tuple(float(v) for v in sampling.cfg_range)
            if sampling.num_inference_steps != 50:
                steps_ovr = int(sampling.num_inference_steps)
        t_seq, guided, _ = build_schedule(sc, steps_ovr, r_ovr, cr_ovr)
        return [float(t) for t in t_seq.tolist()], [bool(g) for g in guided], g_scale

    @torch.no_grad()
    def sample_branch_split(self, vox: torch.Tensor, context: torch.Tensor, *, group=None,
                            sampling: Optional[FlowMatchSamplingParams] = None,
                            generator: Optional[torch.Generator] = None,
                            noise: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One sample on two GPUs (one process each, a two-rank NCCL ``group``; the default
        group when None): in every guided step the conditional NFE runs on group rank 0 and
        the exact 1-token NFE on rank 1 at the same time, and the two velocities are
        exchanged before the shared CFG + Euler update.  Both ranks pass the same voxels and
        context; the noise is rank 0's (``noise`` or a draw from ``generator``), broadcast.
        Both ranks return the same latents ([N, 16] fp32, input voxel order)."""
        import torch.distributed as dist
        from . import distributed as vd
        if self.solver_config.approximate_cfg_cache:
            raise NotImplementedError("the two-GPU branch split runs the exact solver only (cfg_cache_mode 'exact')")
        geom = self._prepare_sample_geometry([vox], context)
        N = geom["N"]
        rank = dist.get_rank(group)
        if rank == 0:
            noise = (torch.randn(N, self.latent_dim, dtype=F32, device=self.device, generator=generator)
                     if noise is None else noise.to(self.device, F32).contiguous())
        else:
            noise = torch.empty(N, self.latent_dim, dtype=F32, device=self.device)
        dist.broadcast(noise, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        tl, guided, g_scale = self._schedule(sampling)
        xt = fk.gather_rows_f32(noise, geom["perm"])

        def nfe(x, t, uncond):
            return self.forward_flow_fast(x, t, context, None, geom, uncond=uncond)

        vd.branch_split_steps(xt, tl, guided, g_scale, nfe, fk.cfg_euler_, group)
        self._b0_share = None
        return fk.unpermute_denorm(xt, geom["up_widx"], self._denorm_scale, self._denorm_shift)

    def _sample_steps(self, geom: Dict[str, Any], context: torch.Tensor, noise: torch.Tensor, tl: List[float],
                      guided: List[bool], g_scale: float) -> torch.Tensor:
        """GPU part of the sampler: Euler + CFG over the schedule, latents in input order.
        With the approximate CFG cache on (``SolverConfig.cfg_cache_mode == "neg_reuse"``), a
        guided step that ``should_eval_uncond`` skips reuses the last unconditional velocity
        (``lib/fast_flow.py:2791-2887``, non-QAOA branch); otherwise every guided step runs both
        NFEs (the exact solver)."""
        xt = fk.gather_rows_f32(noise, geom["perm"])
        main = torch.cuda.current_stream(self.device)
        sc = self.solver_config
        approx = sc.approximate_cfg_cache
        n_guided = sum(1 for g in guided if g)
        last_neg = last_neg_x0 = None
        for i in range(len(guided)):
            both = guided[i] and g_scale > 0
            eval_neg = both and (not approx or last_neg is None or
                                 should_eval_uncond(i, n_guided, sc.cfg_stride, sc.cfg_cache_mode,
                                                    sc.eval_uncond_steps))
            neg = self._negative_stream() if (eval_neg and self.overlap_branches) else main
            if neg is not main:
                neg.wait_stream(main)                     # x_t of this step
                xt.record_stream(neg)
            self._nfe_shared = neg is not main
            v = self.forward_flow_fast(xt, tl[i], context, None, geom)
            vn = None
            if eval_neg:
                with torch.cuda.stream(neg):
                    vn = self.forward_flow_fast(xt, tl[i], context, None, geom, uncond=True)
                if neg is not main:
                    main.wait_stream(neg)
                    vn.record_stream(main)
            t_eval, dt = tl[i], tl[i] - tl[i + 1]
            if both and not eval_neg:
                blend = sc.autotarget_clean_endpoint_blend
                x0 = last_neg_x0 if (blend > 0.0 and t_eval > 0.25) else None
                hf = (sc.fastercache_hf_boost * max(0.0, 1.0 - t_eval)
                      if (sc.fastercache_freq_decoupled_cfg and xt.shape[0] > 1) else 0.0)
                fk.cfg_reuse_euler_(xt, v, last_neg, x0, g_scale, dt, t_eval, blend, hf, sc.cfg_zero_star_projection)
            else:
                if approx and eval_neg:
                    last_neg = vn
                    if sc.autotarget_clean_endpoint_blend > 0.0:
                        last_neg_x0 = fk.neg_endpoint(xt, vn, t_eval)
                fk.cfg_euler_(xt, v, vn, g_scale, dt)
        self._nfe_shared = False
        self._b0_share = None
        return fk.unpermute_denorm(xt, geom["up_widx"], self._denorm_scale, self._denorm_shift)

    def _negative_stream(self) -> torch.cuda.Stream:
        if self._neg_stream is None:
            self._neg_stream = torch.cuda.Stream(self.device)
        return self._neg_stream

    def _capture_sample(self, key, geom, context, noise, tl, guided, g_scale) -> "_SampleGraph":
        """Run the sample once eagerly on a side stream (first-call set-up of every kernel,
        time gates cached), then capture it on the static buffers."""
        ctx = context.clone()
        nz = noise.clone()
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self._sample_steps(geom, ctx, nz, tl, guided, g_scale)
        torch.cuda.current_stream(self.device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = self._sample_steps(geom, ctx, nz, tl, guided, g_scale)
        entry = _SampleGraph(graph, geom, ctx, nz, out)
        self._graphs[key] = entry
        while len(self._graphs) > self.max_graphs:
            self._graphs.popitem(last=False)
        return entry

    @torch.no_grad()
    def warmup(self) -> None:
        """One tiny sample so every kernel (its attributes and tensor maps) is set up before timing."""
        vox = torch.stack(torch.meshgrid(*[torch.arange(4)] * 3, indexing="ij"), -1).reshape(-1, 3)
        dino = torch.zeros(1, 5 + 4, self.arch.dino_dim)
        self.sample_fast([vox.to(self.device)], LatDitConditioning(dino_features=dino.to(self.device)))
        torch.cuda.synchronize(self.device)
