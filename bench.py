"""Benchmark of the sparse-voxel DiT (lat_dit) forward path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Workload (one "step"): one full sample of the 24-block DiT (dim 1536,
12x128 heads, bf16 linears, fp32 ffn_conv) on N=16384 voxels of a sphere
shell (r=36) in 64^3 with a [4101, 1536] N(0,1) image context and the exact
4-step solver (3 CFG-guided steps with the 1-token uncond branch + 1
unguided step = 7 NFE).  Metric: voxel-tokens/s per NFE = 7 * N / step time.
Synthetic data and random-init weights (no checkpoint or dataset here).

With N GPUs (torchrun), every rank runs its own sample per step (weak
scaling) and the latents are gathered to rank 0 over NCCL at the end of each
step; the step time is the max over ranks.  ``--impl reference`` times the
reference algorithm's CPU implementation (the CPU oracle port, fp32) on this
host's cores instead.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

from __graft_entry__ import load_package  # noqa: E402

METRIC = "voxel-tokens/s per DiT NFE"
UNIT = "voxel-tokens/s"
NFE_PER_SAMPLE = 7


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


def _peaks_sustained() -> float:
    """bf16 GEMM rate held for seconds under the power cap (for a kernel timed inside a long step)."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()).get("bf16_tflops_sustained", 1400.0)
    return 1400.0


class ClockSampler:
    """nvidia-smi clock / throttle samples every 200 ms during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def _l2_flush(buf: torch.Tensor):
    buf.add_(1)          # 256 MiB write: larger than the 126 MB L2


CPU_SAMPLE = ("CPU oracle (fp32) at N=16384, L=4101, 12x128: one context block and one plain block of the "
              "conditional NFE and the same two of the exact 1-token NFE; the 7-NFE sample (4 conditional + "
              "3 1-token NFEs, each 8 context + 16 plain blocks) extrapolated from their times")
CPU_BLOCK_KINDS = ("ctx", "plain", "ctx_1tok", "plain_1tok")


class CpuBlocks:
    """The CPU oracle (fp32) on the workload's shapes (N=16384 shell voxels, L=4101 context
    tokens, 12x128 heads): weights of one context block (0) and one plain block (8), the
    voxel set's geometry and the inputs are built once; ``run(kind)`` times one block of the
    conditional NFE ("ctx", "plain") or of the exact 1-token NFE ("ctx_1tok", "plain_1tok")."""

    def __init__(self, threads: int):
        from oracle import model as om
        from vdit.workloads import C4, shell_voxels
        torch.set_num_threads(threads)
        self.om, self.w, D = om, C4(), 1536
        self.cfg = om.ModelConfig(dim=D, head_dim=128, depth=9, cond_depth=8, res=64)
        g = torch.Generator().manual_seed(0)
        self.p = {k: (torch.ones(v) if k.endswith("_scale") or k == "std" else torch.randn(v, generator=g) * 0.02)
                  for k, v in om.param_shapes(self.cfg).items()
                  if ("blocks.0." in k or "blocks.8." in k) and "gates" not in k}
        self.geom = om.build_geometry(shell_voxels(self.w.n, self.w.grid, self.w.radius, 0), self.cfg)
        self.x = torch.randn(self.w.n, D, generator=g)
        self.c = torch.randn(self.w.ctx_tokens, D, generator=g)
        self.c1 = torch.randn(1, D, generator=g)
        self.cpos = om.cond_positions(self.w.ctx_tokens)
        self.gates = {"blocks": [None] * 9, "cond": [None] * 9}
        for b, nc in ((0, 9), (8, 2)):
            self.gates["blocks"][b] = torch.randn(9, D, generator=g) * 0.1
            self.gates["cond"][b] = torch.randn(nc, D, generator=g) * 0.1

    def run(self, kind: str) -> float:
        om, p, cfg, x, gates, geom = self.om, self.p, self.cfg, self.x, self.gates, self.geom
        fn = {"ctx": lambda: om.block_forward(p, cfg, 0, x, self.c, gates, geom, self.cpos),
              "plain": lambda: om.block_forward(p, cfg, 8, x, self.c, gates, geom, None),
              "ctx_1tok": lambda: om.block_forward_1tok(p, cfg, 0, x, self.c1, None, gates, geom),
              "plain_1tok": lambda: om.block_forward_1tok(p, cfg, 8, x, self.c1, None, gates, geom)}[kind]
        t0 = time.perf_counter()
        with torch.no_grad():
            fn()
        return time.perf_counter() - t0

    def value(self, t: dict) -> float:
        """Voxel-tokens/s per NFE of a 7-NFE sample from the block times ``t`` (seconds per
        kind): 4 x (8 context + 16 plain blocks) + 3 x (8 + 16 blocks of the 1-token branch),
        the GPU arm's mix."""
        t_sample = 4 * (8 * t["ctx"] + 16 * t["plain"]) + 3 * (8 * t["ctx_1tok"] + 16 * t["plain_1tok"])
        return NFE_PER_SAMPLE * self.w.n / t_sample


def cpu_baseline_sample(threads: int):
    """One CPU sample of the four block kinds, each run once.  Returns (voxel-tokens/s per
    NFE, seconds of CPU work)."""
    cb = CpuBlocks(threads)
    t = {k: cb.run(k) for k in CPU_BLOCK_KINDS}
    return cb.value(t), sum(t.values())


def run_reference(args):
    """--impl reference: the reference algorithm on the host CPU (oracle port).  Only the
    workload generator of the package is used (the same voxel sets as the GPU arm).  The
    blocks are built once; step i times one block of kind i mod 4 (the warm-up steps run the
    same rotation untimed), and the line's value combines the median time of each kind
    (kinds that no timed step reached are timed once more at the end)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    load_package()
    threads = os.cpu_count() or 1
    cb = CpuBlocks(threads)
    for i in range(args.warmup):
        cb.run(CPU_BLOCK_KINDS[i % 4])
    per_kind = {k: [] for k in CPU_BLOCK_KINDS}
    times = []
    for i in range(args.steps):
        dt = cb.run(CPU_BLOCK_KINDS[i % 4])
        per_kind[CPU_BLOCK_KINDS[i % 4]].append(dt)
        times.append(dt)
    for k, v in per_kind.items():
        if not v:
            v.append(cb.run(k))
    value = float(cb.value({k: statistics.median(v) for k, v in per_kind.items()}))
    sample = CPU_SAMPLE + "; one block per step, in rotation over the four kinds"
    w = cb.w
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * statistics.median(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "C4 full 24-block DiT, N=16384 shell r=36 in 64^3, 4101x1536 context, 12x128 heads",
                   "global_batch": 1, "seq_len": w.n},
        "block_seconds": {k: statistics.median(v) for k, v in per_kind.items()},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def attention_roofline(w, runner, reps: int = 20):
    """Average duration of the window self-attention kernel on the workload's shapes
    (N=16384 in four 4096-voxel windows, 12x128 heads), CUDA events on its stream."""
    from vdit import fast_kernels as fk
    D, H, HD = w.arch.dim, w.arch.heads, w.arch.head_dim
    g = torch.Generator(device="cuda").manual_seed(1)
    qkv = torch.randn(w.n, 3 * D, device="cuda", generator=g).to(torch.bfloat16)
    out = torch.empty(w.n, D, device="cuda", dtype=torch.bfloat16)
    cu = list(range(0, w.n, 4096)) + [w.n]
    for _ in range(3):
        fk.attention(qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:], cu, cu, H, HD, out=out)
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(s)
    for _ in range(reps):
        fk.attention(qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:], cu, cu, H, HD, out=out)
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    flops = sum(4.0 * (cu[i + 1] - cu[i]) ** 2 * D for i in range(len(cu) - 1))
    return flops, ms


def vendor_attention_bars(w, reps: int = 20) -> dict:
    """Library attention on the same window self-attention shapes (four 4096-voxel windows,
    12 x 128 heads, bf16), reported beside the kernel only: torch SDPA with the cuDNN and
    the flash backends, and the flash_attn package's varlen packed-QKV entry point (the
    reference's attention backend, ``lib/fast_kernels.py:1538-1587``).  CUDA events; a
    backend that does not run on this GPU is reported with its error."""
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel
    D, H, HD = w.arch.dim, w.arch.heads, w.arch.head_dim
    nwin = w.n // 4096
    g = torch.Generator(device="cuda").manual_seed(1)
    q, k, v = (torch.randn(nwin, H, 4096, HD, device="cuda", generator=g).to(torch.bfloat16) for _ in range(3))
    flops = 4.0 * nwin * 4096 * 4096 * D
    s = torch.cuda.current_stream()

    def timed(fn):
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(s)
        for _ in range(reps):
            fn()
        e1.record(s)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        return {"ms_per_launch": ms, "tflops": flops / ms / 1e9}

    out = {}
    for name, backend in (("sdpa_cudnn", SDPBackend.CUDNN_ATTENTION), ("sdpa_flash", SDPBackend.FLASH_ATTENTION)):
        try:
            with sdpa_kernel([backend]):
                out[name] = timed(lambda: F.scaled_dot_product_attention(q, k, v))
        except Exception as exc:  # a backend without sm_100 support
            out[name] = {"error": f"{type(exc).__name__}: {str(exc)[:160]}"}
    try:
        from flash_attn import flash_attn_varlen_qkvpacked_func
        qkv = torch.stack([q, k, v], 2).permute(0, 3, 2, 1, 4).reshape(nwin * 4096, 3, H, HD).contiguous()
        cu = torch.arange(0, nwin + 1, device="cuda", dtype=torch.int32) * 4096
        out["flash_attn_varlen_qkvpacked"] = timed(lambda: flash_attn_varlen_qkvpacked_func(qkv, cu, 4096))
    except Exception as exc:
        out["flash_attn_varlen_qkvpacked"] = {"error": f"{type(exc).__name__}: {str(exc)[:160]}"}
    return out


def dwconv_roofline(w, reps: int = 20):
    """Average duration of the depthwise conv + SwiGLU kernel on the workload's shapes
    (N=16384 shell voxels, 7680 -> 3840 channels), CUDA events on its stream.
    Algorithmic bytes: read N*2F*2 + write N*F*2 + weights 27*2F*4 + indices N*27*4."""
    from vdit import fast_kernels as fk
    from vdit.workloads import shell_voxels
    vox = torch.from_numpy(shell_voxels(w.n, w.grid, w.radius, 0)).cuda()
    _, _, hc = fk.lex_perm(vox)
    idx = fk.build_conv_indices_fast(hc, already_sorted=True)[0]
    f2 = 2 * w.arch.ffn_dim
    g = torch.Generator(device="cuda").manual_seed(2)
    h = torch.randn(w.n, f2, device="cuda", generator=g).to(torch.bfloat16)
    cw = 0.05 * torch.randn(27, f2, device="cuda", generator=g)
    cb = torch.zeros(f2, device="cuda")
    fwd, _ = fk.hilbert4_orders(hc, 1024)
    plan = fk.build_conv_plan([idx], fwd[0])
    byts = w.n * f2 * 2 + w.n * (f2 // 2) * 2 + 27 * f2 * 4 + w.n * 27 * 4
    s = torch.cuda.current_stream()

    def timed(fn):
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(s)
        for _ in range(reps):
            fn()
        e1.record(s)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    ms_gather = timed(lambda: fk.fast_sparse_conv3d(h, cw, cb, [idx], fuse_swiglu=True))
    ms_planned = timed(lambda: fk.fast_sparse_conv3d_swiglu_planned(h, cw, cb, plan))
    return byts, ms_planned, ms_gather


def qknorm_bench(w, reps: int = 20):
    """QK-RMSNorm + 3D RoPE + Hilbert gather on the workload's shapes (N=16384, 12x128).
    Algorithmic bytes: read + write of [N, 3, H, HD] bf16 plus the gather index."""
    from vdit import fast_kernels as fk
    from vdit.workloads import shell_voxels
    vox = torch.from_numpy(shell_voxels(w.n, w.grid, w.radius, 0)).cuda()
    _, _, hc = fk.lex_perm(vox)
    fwd, _ = fk.hilbert4_orders(hc, 1024)
    D, H, HD = w.arch.dim, w.arch.heads, w.arch.head_dim
    g = torch.Generator(device="cuda").manual_seed(4)
    qkv = torch.randn(w.n, 3 * D, device="cuda", generator=g).to(torch.bfloat16)
    qs = torch.ones(H, HD, device="cuda")
    cos, sin = fk.precompute_rope_3d_table(64, 128.0, HD, device="cuda")
    out = torch.empty_like(qkv)
    for _ in range(3):
        fk.fused_qknorm_rope3d_gather(qkv, qs, qs, cos, sin, hc, fwd[0], H, HD, out=out)
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(s)
    for _ in range(reps):
        fk.fused_qknorm_rope3d_gather(qkv, qs, qs, cos, sin, hc, fwd[0], H, HD, out=out)
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    byts = 2 * w.n * 3 * D * 2 + w.n * 8
    return {"kernel": "qknorm_rope_kernel<0>", "ms_per_launch": ms, "gbs": byts / ms / 1e6}


def gate_add_bench(w, reps: int = 20):
    """Gate-add + LayerNorm + AdaLN modulation on the workload's shapes (N=16384, D=1536).
    Algorithmic bytes: read x and h, write x and the modulated copy (4*N*D*2)."""
    from vdit import fast_kernels as fk
    D = w.arch.dim
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(w.n, D, device="cuda", generator=g).to(torch.bfloat16)
    h = torch.randn(w.n, D, device="cuda", generator=g).to(torch.bfloat16)
    gt, s1, sh = [torch.randn(D, device="cuda", generator=g) * 0.1 for _ in range(3)]
    mod = torch.empty_like(x)
    for _ in range(3):
        fk.fast_gate_add_and_modulate(x, h, gt, s1, sh, out=mod)
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(s)
    for _ in range(reps):
        fk.fast_gate_add_and_modulate(x, h, gt, s1, sh, out=mod)
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    return {"kernel": "gate_add_modulate", "ms_per_launch": ms, "gbs": 4 * w.n * D * 2 / ms / 1e6}


def hbm_bench(w, reps: int = 10):
    """The HBM-bound kernels of the path on the workload's shapes (N=16384 voxels, D=1536,
    12x128 heads; geometry at N=262144 uniform voxels in 128^3).  Each launch is timed
    alone with CUDA events after a 256 MiB L2 flush; median of ``reps`` launches after two
    warm-up launches.  Algorithmic bytes (each tensor counted once):
    gate-add + LN + AdaLN 4*N*D*2; LN + AdaLN 2*N*D*2; QK-norm/RoPE/gather 2*3*N*D*2 + 8N;
    out-modulate-unpatchify and the unpatchify projection N*D*2 + N*16*4; patchify N*16*4 + N*D*2; single query over
    formed K/V 2*N*D*2; single query over the voxel rows N*D*2 + 2*D*D*2 (W_k, W_v)."""
    from vdit import fast_kernels as fk
    from vdit.workloads import shell_voxels, uniform_voxels
    hbm, _, kind = _peaks()
    n, D, H, HD = w.n, w.arch.dim, w.arch.heads, w.arch.head_dim
    g = torch.Generator(device="cuda").manual_seed(11)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream()

    def timed(fn):
        for _ in range(2):
            fn()
        ms = []
        for _ in range(reps):
            _l2_flush(flush)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            fn()
            e1.record(s)
            torch.cuda.synchronize()
            ms.append(e0.elapsed_time(e1))
        return statistics.median(ms)

    def row(name, kernel, fn, byts=None):
        ms = timed(fn)
        r = {"op": name, "kernel": kernel, "ms": round(ms, 4)}
        if byts is not None:
            r.update({"bytes": int(byts), "gbs": round(byts / ms / 1e6, 1),
                      "frac_hbm": round(byts / ms / 1e6 / hbm, 3), "peak": f"{hbm} GB/s ({kind})"})
        return r

    bf = torch.bfloat16
    x = torch.randn(n, D, device="cuda", generator=g).to(bf)
    h = torch.randn(n, D, device="cuda", generator=g).to(bf)
    gt, s1, sh, g2 = [torch.randn(D, device="cuda", generator=g) * 0.1 for _ in range(4)]
    crow = torch.randn(D, device="cuda", generator=g).to(bf)
    mod = torch.empty_like(x)
    out = []
    out.append(row("gate-add + LN + AdaLN", "gate_add_modulate_staged_kernel",
                   lambda: fk.fast_gate_add_and_modulate(x, h, gt, s1, sh, out=mod), 4 * n * D * 2))
    out.append(row("LN + AdaLN", "gate_add_modulate_staged_kernel (no residual)",
                   lambda: fk.fast_modulate(x, None, s1, sh, out=mod), 2 * n * D * 2))
    out.append(row("two gate-adds + LN + AdaLN (1-token branch)", "gate_add_modulate_staged_kernel (c2, g2)",
                   lambda: fk.fast_gate_add2_and_modulate(x, h, gt, crow, g2, s1, sh, out=mod), 4 * n * D * 2))
    vox = torch.from_numpy(shell_voxels(n, w.grid, w.radius, 0)).cuda()
    _, _, hc = fk.lex_perm(vox)
    fwd, _ = fk.hilbert4_orders(hc, 1024)
    cos, sin = fk.precompute_rope_3d_table(w.grid, 128.0, HD, device="cuda")
    qkv = torch.randn(n, 3 * D, device="cuda", generator=g).to(bf)
    qkv_o = torch.empty_like(qkv)
    qs = torch.ones(H, HD, device="cuda")
    out.append(row("QK-RMSNorm + RoPE3D + window gather (separate pass)", "qknorm_rope_kernel<0>",
                   lambda: fk.fused_qknorm_rope3d_gather(qkv, qs, qs, cos, sin, hc, fwd[0], H, HD, out=qkv_o),
                   2 * 3 * n * D * 2 + 8 * n))
    wu = torch.randn(16, D, device="cuda", generator=g) * 0.02
    out.append(row("out LN + AdaLN + unpatchify (one call)", "out_unpatchify_kernel<6>",
                   lambda: fk.fast_out_modulate_unpatchify(x, None, s1, sh, wu), n * D * 2 + n * 16 * 4))
    wu3 = fk.split_weight3(wu)
    out.append(row("unpatchify projection of the modulated rows (the runner's path)", "unpatchify_project_kernel",
                   lambda: fk.unpatchify_project(mod, wu3), n * D * 2 + n * 16 * 4))
    xt = torch.randn(n, 16, device="cuda", generator=g)
    wp = torch.randn(D, 16, device="cuda", generator=g) * 0.02
    out.append(row("patchify", "patchify_kernel", lambda: fk.patchify(xt, wp), n * 16 * 4 + n * D * 2))
    q = torch.randn(D, device="cuda", generator=g)
    kv = torch.randn(n, 2 * D, device="cuda", generator=g).to(bf)
    out.append(row("single query over formed K/V", "attn1q_partial_kernel + attn1q_combine_kernel",
                   lambda: fk.attention_1q(q, kv, H, HD), 2 * n * D * 2))
    wkv = (torch.randn(2 * D, D, device="cuda", generator=g) * 0.02).to(bf)
    bkv = (torch.randn(2 * D, device="cuda", generator=g) * 0.02).to(bf)
    out.append(row("single query over the voxel rows (K/V not formed)", "wide1q_fold/partial/merge/project",
                   lambda: fk.attention_1q_wide(q, x, wkv, bkv, H, HD), n * D * 2 + 2 * D * D * 2))
    # per-sample geometry at the largest C2 size (sort-dominated; times only)
    big = torch.from_numpy(uniform_voxels(262144, 128, 1)).cuda()
    _, _, hcb = fk.lex_perm(big)
    out.append(row("lexicographic order (N=262144)", "vdit_lex_perm", lambda: fk.lex_perm(big)))
    out.append(row("four Hilbert orders + windows (N=262144)", "vdit_hilbert4_orders",
                   lambda: fk.hilbert4_orders(hcb, 1024)))
    out.append(row("conv_indices (N=262144)", "conv_indices_kernel",
                   lambda: fk.build_conv_indices_fast(hcb, already_sorted=True)))
    return out


def gemm_bench(w, reps: int = 20):
    """The block linears of the workload (M = N voxels or the L context rows, bf16
    in/out, fp32 accumulation): the tcgen05 GEMM beside cuBLAS (``F.linear``), same
    inputs, CUDA events.  FLOPs 2*M*K*Nout per launch."""
    import torch.nn.functional as F
    from vdit import fast_kernels as fk
    D = w.arch.dim
    F2 = 2 * w.arch.ffn_dim
    shapes = [("to_qkv", w.n, D, 3 * D), ("to_out", w.n, D, D), ("ffn0", w.n, D, F2),
              ("ffn1", w.n, F2 // 2, D), ("cond_to_qkv", w.ctx_tokens, D, 3 * D),
              ("cond_to_out", w.ctx_tokens, D, D), ("cond_to_kv_cross", w.ctx_tokens, D, 2 * D),
              ("cond_ffn0", w.ctx_tokens, D, F2), ("cond_ffn1", w.ctx_tokens, F2 // 2, D),
              ("image_map", w.ctx_tokens, w.arch.dino_dim, D)]
    g = torch.Generator(device="cuda").manual_seed(9)
    s = torch.cuda.current_stream()
    res = []
    for name, m, k, n in shapes:
        a = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
        wt = (0.02 * torch.randn(n, k, device="cuda", generator=g)).to(torch.bfloat16)
        b = (0.02 * torch.randn(n, device="cuda", generator=g)).to(torch.bfloat16)
        out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
        row = {"gemm": name, "m": m, "k": k, "n": n}
        for impl, fn in (("tcgen05", lambda: fk.linear(a, wt, b, out=out)), ("cublas", lambda: F.linear(a, wt, b))):
            for _ in range(3):
                fn()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record(s)
            for _ in range(reps):
                fn()
            e1.record(s)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / reps
            row[impl + "_ms"] = round(ms, 4)
            row[impl + "_tflops"] = round(2 * m * k * n / ms / 1e9, 1)
            # the same launches replayed from a CUDA graph: device time without host launch gaps
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for _ in range(reps):
                    fn()
            graph.replay()
            torch.cuda.synchronize()
            e0.record(s)
            graph.replay()
            e1.record(s)
            torch.cuda.synchronize()
            row[impl + "_graph_ms"] = round(e0.elapsed_time(e1) / reps, 4)
            del graph
        ref = F.linear(a, wt, b).float()
        row["rel_l2_vs_cublas"] = float((fk.linear(a, wt, b).float() - ref).norm() / ref.norm())
        res.append(row)
    # the self-attention qkv with QK-norm, RoPE3D and the window-order scatter in the epilogue,
    # against cuBLAS followed by the separate QK-norm / RoPE / gather pass
    from vdit.workloads import shell_voxels
    H, HD = w.arch.heads, w.arch.head_dim
    vox = torch.from_numpy(shell_voxels(w.n, w.grid, w.radius, 0)).cuda()
    _, _, hc = fk.lex_perm(vox)
    fwd, bwd = fk.hilbert4_orders(hc, w.grid)
    fwd, bwd = fwd[0].contiguous(), bwd[0].contiguous()
    cos, sin = fk.precompute_rope_3d_table(w.grid, 128.0, HD, device="cuda")
    a = torch.randn(w.n, D, device="cuda", generator=g).to(torch.bfloat16)
    wt = (0.02 * torch.randn(3 * D, D, device="cuda", generator=g)).to(torch.bfloat16)
    b = (0.02 * torch.randn(3 * D, device="cuda", generator=g)).to(torch.bfloat16)
    qs, ks = 1 + 0.1 * torch.randn(D, device="cuda", generator=g), 1 + 0.1 * torch.randn(D, device="cuda", generator=g)
    out = torch.empty(w.n, 3 * D, device="cuda", dtype=torch.bfloat16)
    row = {"gemm": "to_qkv + QK-norm/RoPE3D/window scatter", "m": w.n, "k": D, "n": 3 * D}
    impls = (("fused_epilogue", lambda: fk.linear_qkv_rope3d(a, wt, b, qs, ks, cos, sin, hc, bwd, H, HD, out=out)),
             ("cublas_then_qknorm", lambda: fk.fused_qknorm_rope3d_gather(F.linear(a, wt, b), qs, ks, cos, sin, hc,
                                                                         fwd, H, HD, out=out)))
    for impl, fn in impls:
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(s)
        for _ in range(reps):
            fn()
        e1.record(s)
        torch.cuda.synchronize()
        row[impl + "_ms"] = round(e0.elapsed_time(e1) / reps, 4)
    res.append(row)
    return res


def dense_conv_bench(reps: int = 5):
    """C3: dense 27-tap sparse conv, N=65536 voxels of a sphere shell (r=56) in 128^3,
    features [N,1536] bf16, weights [27,1536,1536], fp32 accumulation.  FLOPs are
    reported per present neighbour (2*nnz*Cin*Cout) and for all 27 taps."""
    from vdit import fast_kernels as fk
    from vdit.workloads import shell_voxels
    n, cin, cout = 65536, 1536, 1536
    vox = torch.from_numpy(shell_voxels(n, 128, 56.0, 3)).cuda()
    _, _, hc = fk.lex_perm(vox)
    idx = fk.build_conv_indices_fast(hc, already_sorted=True)[0]
    nnz = int((idx >= 0).sum())
    g = torch.Generator(device="cuda").manual_seed(3)
    f = torch.randn(n, cin, device="cuda", generator=g).to(torch.bfloat16)
    wt = (0.02 * torch.randn(27, cout, cin, device="cuda", generator=g)).to(torch.bfloat16)
    b = torch.zeros(cout, device="cuda")
    for _ in range(2):
        fk.dense_sparse_conv3d(f, wt, b, [idx])
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(s)
    for _ in range(reps):
        fk.dense_sparse_conv3d(f, wt, b, [idx])
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    return {"kernel": "dense_conv27_kernel", "ms_per_launch": ms, "nnz": nnz,
            "tflops_nnz": 2.0 * nnz * cin * cout / ms / 1e9, "tflops_dense27": 2.0 * 27 * n * cin * cout / ms / 1e9}


def branch_split_bench(w, reps: int = 3):
    """One C4 sample on two GPUs (torchrun, two ranks): the branch split (conditional NFE on
    rank 0, exact 1-token NFE on rank 1, velocities exchanged over NCCL in every guided
    step) against the same sample on rank 0 alone.  Latency per sample from CUDA events,
    max over the two ranks."""
    import torch.distributed as dist
    from vdit.fast_flow import OptimizedLatDitRunner
    from vdit.fast_sampler import SolverConfig
    from vdit.model import LatDitModel
    rank = dist.get_rank()
    dev = torch.device("cuda", torch.cuda.current_device())
    model = LatDitModel.random(w.arch, seed=0, device=dev)
    solver = SolverConfig(num_inference_steps=4, n_guided_steps=3, n_unguided_steps=1, guidance_scale=w.guidance)
    runner = OptimizedLatDitRunner(model, solver, device=dev)
    inp = w.inputs(seed=100, device=dev)                 # the same sample on both ranks
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    s = torch.cuda.current_stream()

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        dist.barrier()
        tot = 0.0
        for _ in range(reps):
            _l2_flush(flush)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            fn()
            e1.record(s)
            torch.cuda.synchronize()
            tot += e0.elapsed_time(e1)
        t = torch.tensor([tot / reps], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    split_ms = timed(lambda: runner.sample_branch_split(inp["vox"], inp["context"], noise=inp["noise"]))
    one = runner.sample_with_context(inp["vox"], inp["context"], noise=inp["noise"])
    two = runner.sample_branch_split(inp["vox"], inp["context"], noise=inp["noise"])
    same = float((one - two).float().norm() / one.float().norm())
    one_ms = timed(lambda: runner.sample_with_context(inp["vox"], inp["context"], noise=inp["noise"])
                   if rank == 0 else None)
    return {"mode": "branch_split", "n_gpus": 2, "voxels": w.n, "split_ms_per_sample": split_ms,
            "one_gpu_ms_per_sample": one_ms, "speedup": one_ms / split_ms, "rel_l2_split_vs_one_gpu": same}


def graph_bench(w, reps: int = 5):
    """Sample latency, eager vs CUDA-graph replay, on the workload's model at N = 4632
    (the size of the smallest public-test voxel set) and at the workload's N."""
    from vdit.fast_flow import OptimizedLatDitRunner
    from vdit.fast_sampler import SolverConfig
    from vdit.model import LatDitModel
    from vdit.runtime import LatDitConditioning
    from vdit.workloads import shell_voxels
    dev = torch.device("cuda", torch.cuda.current_device())
    model = LatDitModel.random(w.arch, seed=0, device=dev)
    solver = SolverConfig(num_inference_steps=4, n_guided_steps=3, n_unguided_steps=1, guidance_scale=w.guidance)
    runner = OptimizedLatDitRunner(model, solver, device=dev)
    g = torch.Generator().manual_seed(9)
    dino = torch.randn(1, w.ctx_tokens, w.arch.dino_dim, generator=g).to(dev, torch.float16)
    cond = LatDitConditioning(dino_features=dino)
    out = {"kernel": "sample (7 NFE)", "reps": reps}
    for n, radius in ((4632, 30.0), (w.n, w.radius)):
        vox = torch.from_numpy(shell_voxels(n, w.grid, radius, 1)).to(dev)
        noise = torch.randn(len(vox), 16, generator=g).to(dev)
        res = {}
        for mode in (False, True):
            runner.cuda_graph = mode
            for _ in range(2):
                runner.sample_fast([vox], cond, noise=noise)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                runner.sample_fast([vox], cond, noise=noise)
            e1.record()
            torch.cuda.synchronize()
            res["graph_ms" if mode else "eager_ms"] = e0.elapsed_time(e1) / reps
        out[f"n{len(vox)}"] = res
    return out


def c5_bench(rank: int, ws: int, dev, dist, samples: int = 0, steps: int = 1, warmup: int = 1,
             model=None) -> dict:
    """The sharded batch: ``samples`` C5 samples (N=32768 ellipsoid-union voxels in 128^3,
    default 16) split round-robin over the ranks, latents gathered to rank 0 over NCCL.
    One step processes the whole batch once (strong scaling: the batch is fixed, the
    ranks share it); device time from CUDA events, max over ranks, with each rank's own
    time and the gather's share.  ``model`` (a LatDitModel on ``dev``) reuses its weights."""
    from vdit import _lib
    from vdit import distributed as vd
    from vdit.fast_sampler import SolverConfig
    from vdit.model import LatDitModel
    from vdit.solution import Solution
    from vdit.workloads import C5
    w = C5()
    samples = samples or w.samples
    if samples % ws:
        raise SystemExit(f"{samples} C5 samples do not split evenly over {ws} ranks")
    model = LatDitModel(w.arch, model.state) if model is not None else LatDitModel.random(w.arch, seed=0, device=dev)
    solver = SolverConfig(num_inference_steps=4, n_guided_steps=3, n_unguided_steps=1, guidance_scale=w.guidance)
    runner = Solution(model, solver_config=solver, device=dev).runner
    inps = [w.inputs(seed=500 + i, device=dev) for i in range(rank, samples, ws)]
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    s = torch.cuda.current_stream()
    gather_evs = []

    def step(timed_gather=False):
        lats = [runner.sample_with_context(i["vox"], i["context"], noise=i["noise"]) for i in inps]
        if dist is not None:
            if timed_gather:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(s)
            vd.gather_latents(lats, rank, ws)
            if timed_gather:
                e1.record(s)
                gather_evs.append((e0, e1))

    for _ in range(warmup):
        step()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    launches0 = _lib.launch_count()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(torch.cuda.current_device()) as clk:
        for i in range(steps):
            _l2_flush(flush)
            evs[i][0].record(s)
            step(timed_gather=True)
            evs[i][1].record(s)
        torch.cuda.synchronize()
    launches = (_lib.launch_count() - launches0) // max(steps, 1)
    mine = sum(a.elapsed_time(b) for a, b in evs) / steps
    gather_ms = sum(a.elapsed_time(b) for a, b in gather_evs) / steps if gather_evs else 0.0
    per_rank = torch.tensor([mine, gather_ms], device=dev)
    if dist is not None:
        allr = [torch.zeros_like(per_rank) for _ in range(ws)]
        dist.barrier()
        dist.all_gather(allr, per_rank)
        allr = torch.stack(allr).cpu()
    else:
        allr = per_rank.cpu()[None]
    ms_step = float(allr[:, 0].max())
    assert _lib.device_error() == 0, "device error word set during the benchmark"
    del runner
    return {
        "metric": METRIC, "value": samples * NFE_PER_SAMPLE * w.n / (ms_step / 1e3), "unit": UNIT,
        "samples_per_s": samples / (ms_step / 1e3), "ms_per_step": ms_step, "steps": steps, "warmup": warmup,
        "ms_per_sample": ms_step * ws / samples, "scaling": "strong",
        "rank_ms_min": float(allr[:, 0].min()), "rank_ms_max": ms_step,
        "gather_ms_max": float(allr[:, 1].max()),
        "config": {"workload": f"C5 sharded batch: {samples} samples x N={w.n} (1-3 ellipsoid shells in "
                               f"{w.grid}^3), 24-block DiT, 4101x1536 context, 4-step exact solver = 7 NFE each",
                   "global_batch": samples, "seq_len": w.n, "parallelism": f"samples x{ws}",
                   "l2": "256 MiB L2 flush before every timed step"},
        "gpu_launches": int(launches), "clocks": clk.summary()}


def cfg_cache_bench(w, reps: int = 5) -> dict:
    """Quality and speed of the approximate CFG cache on the C4 workload (the reference's
    "neg_reuse" defaults: unconditional NFE at guided steps 0 and 2 only, 6 NFE per sample
    instead of 7) against the exact solver: ms per sample (CUDA events, L2 flushed before each
    sample) and the relative L2 distance of the final latents from the exact ones."""
    from vdit.fast_flow import OptimizedLatDitRunner
    from vdit.fast_sampler import SolverConfig
    from vdit.model import LatDitModel
    dev = torch.device("cuda", torch.cuda.current_device())
    model = LatDitModel.random(w.arch, seed=0, device=dev)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    s = torch.cuda.current_stream()
    out = {"workload": "C4 (24 blocks, N=16384, 4101 context tokens, CFG 3.0)"}
    lats = {}
    for mode in ("exact", "neg_reuse"):
        solver = SolverConfig(num_inference_steps=4, n_guided_steps=3, n_unguided_steps=1, guidance_scale=w.guidance)
        if mode == "neg_reuse":
            solver.enable_approximate_cfg_cache()
        runner = OptimizedLatDitRunner(model, solver, device=dev)
        ms = []
        for seed in range(3):
            inp = w.inputs(seed=100 + seed, device=dev)
            runner.sample_with_context(inp["vox"], inp["context"], noise=inp["noise"])
            torch.cuda.synchronize()
            lat = None
            for _ in range(reps):
                flush.add_(1)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(s)
                lat = runner.sample_with_context(inp["vox"], inp["context"], noise=inp["noise"])
                e1.record(s)
                torch.cuda.synchronize()
                ms.append(e0.elapsed_time(e1))
            lats[(mode, seed)] = lat.float().cpu()
        out[mode] = {"ms_per_sample": statistics.median(ms), "nfe_per_sample": 7 if mode == "exact" else 6}
        del runner
    errs = [float((lats[("neg_reuse", k)] - lats[("exact", k)]).norm() / lats[("exact", k)].norm()) for k in range(3)]
    out["latent_rel_l2_vs_exact"] = errs
    out["speedup"] = out["exact"]["ms_per_sample"] / out["neg_reuse"]["ms_per_sample"]
    return out


def kernel_table(timer: dict, hbm_peak: float, tensor_peak: float, peak_kind: str, solo: dict = None) -> list:
    """Per kernel class: launches, average CUDA-event duration, algorithmic FLOPs or bytes
    per launch and the fraction of the measured peak (sustained bf16 GEMM rate for
    tensor-core classes, HBM copy bandwidth for byte-bound ones).  `timer` holds the launches
    of one whole sample run right after the timed steps, where a guided step runs its two NFEs
    on two streams that share the GPU; `solo`, when given, the same classes from one NFE of
    each branch with every kernel alone on the GPU (`solo_ms_per_launch`, `solo_frac`)."""
    from vdit.fast_flow import KERNEL_CLASSES

    def rate(kind, ev):
        ms = statistics.fmean(a.elapsed_time(b) for a, b, _, _ in ev)
        units = statistics.fmean(u for _, _, u, _ in ev)
        bound = KERNEL_CLASSES.get(kind, "tensor")
        if bound == "tensor":
            return bound, ms, units, units / (ms / 1e3) / 1e12, "TFLOP/s", tensor_peak
        return bound, ms, units, units / (ms / 1e3) / 1e9, "GB/s", hbm_peak

    rows = []
    for kind, ev in timer.items():
        if not ev:
            continue
        bound, ms, units, ach, unit, peak = rate(kind, ev)
        row = {"kernel": kind, "bound": bound, "launches": len(ev), "ms_per_launch": ms,
               "units_per_launch": units, "achieved": ach, "unit": unit, "peak": peak, "frac": ach / peak,
               "total_ms": ms * len(ev),
               "peak_kind": f"{peak_kind} {'sustained bf16' if bound == 'tensor' else 'HBM copy'}"}
        if solo and solo.get(kind):
            _, sms, _, sach, _, _ = rate(kind, solo[kind])
            row.update(solo_ms_per_launch=sms, solo_achieved=sach, solo_frac=sach / peak)
        rows.append(row)
    rows.sort(key=lambda r: -r["total_ms"])
    return rows


def attention_traffic():
    """DRAM bytes per launch of the window self-attention kernel from the committed ncu
    capture, when it was taken on the current kernel source (its SHA-256 is recorded with
    it); None otherwise."""
    import hashlib
    tp = ROOT / "profiles" / "attention_traffic.json"
    if not tp.exists():
        return None
    d = json.loads(tp.read_text())
    src = ROOT / "3d-dit-distillation_b200" / "csrc" / "attention.cu"
    if d.get("source_sha256") != hashlib.sha256(src.read_bytes()).hexdigest():
        return None
    return d.get("dram_bytes_per_launch")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="vdit", choices=["vdit", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", action="store_true",
                    help="one warm-up sample, then one sample inside the NVTX range 'profile_step' (for ncu)")
    ap.add_argument("--only", choices=["attention", "dwconv", "dense_conv", "qknorm", "gate_add", "graph", "gemm", "branch_split",
                                       "c5", "hbm", "cfg_cache"], default=None,
                    help="run only one kernel on the workload's shapes (small ncu case); c5: the sharded batch")
    ap.add_argument("--samples", type=int, default=0, help="--only c5: batch size (default 16)")
    ap.add_argument("--c5-steps", type=int, default=1, help="timed passes of the C5 batch in the default run")
    ap.add_argument("--no-c5", action="store_true", help="skip the C5 sharded batch in the default run")
    ap.add_argument("--reps", type=int, default=10, help="--only hbm: timed launches per kernel")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)

    vdit = load_package()
    from vdit import _lib
    from vdit.fast_flow import OptimizedLatDitRunner
    from vdit.fast_sampler import SolverConfig
    from vdit.model import LatDitModel
    from vdit.runtime import LatDitConditioning
    from vdit.solution import Solution
    from vdit.workloads import C4

    from vdit import distributed as vd
    rank, ws, local = vd.init_from_env("nccl", timeout_s=120)
    dist = torch.distributed if ws > 1 else None
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    w = C4()
    if args.only == "c5":
        r = c5_bench(rank, ws, dev, dist, samples=args.samples, steps=args.steps, warmup=args.warmup)
        if rank == 0:
            print(json.dumps(dict(r, n_gpus=ws, higher_is_better=True, dtype="bf16",
                                  data="synthetic (seeded ellipsoid-union voxels, N(0,1) context, random-init "
                                       "weights)")), flush=True)
        if dist is not None:
            dist.destroy_process_group()
        return
    if args.only == "attention":
        flops, ms = attention_roofline(w, None)
        print(json.dumps({"kernel": "attention_kernel<128>", "ms_per_launch": ms, "tflops": flops / ms / 1e9,
                          "library": vendor_attention_bars(w)}))
        return
    if args.only == "cfg_cache":
        print(json.dumps(cfg_cache_bench(w)))
        return
    if args.only == "qknorm":
        print(json.dumps(qknorm_bench(w)))
        return
    if args.only == "gate_add":
        print(json.dumps(gate_add_bench(w)))
        return
    if args.only == "hbm":
        for r in hbm_bench(w, reps=args.reps):
            print(json.dumps(r))
        return
    if args.only == "branch_split":
        if ws != 2:
            raise SystemExit("--only branch_split runs under torchrun with two ranks")
        r = branch_split_bench(w)
        if rank == 0:
            print(json.dumps(r))
        dist.destroy_process_group()
        return
    if args.only == "gemm":
        for row in gemm_bench(w):
            print(json.dumps(row))
        return
    if args.only == "graph":
        print(json.dumps(graph_bench(w)))
        return
    if args.only == "dense_conv":
        print(json.dumps(dense_conv_bench()))
        return
    if args.only == "dwconv":
        byts, ms, ms_gather = dwconv_roofline(w)
        print(json.dumps({"kernel": "dwconv_planned_kernel (fused SwiGLU)", "ms_per_launch": ms,
                          "gbs": byts / ms / 1e6, "gather_kernel_ms": ms_gather}))
        return
    model = LatDitModel.random(w.arch, seed=0, device=dev)
    solver = SolverConfig(num_inference_steps=4, n_guided_steps=3, n_unguided_steps=1, guidance_scale=w.guidance)
    sol = Solution(model, solver_config=solver, device=dev)
    runner: OptimizedLatDitRunner = sol.runner
    inp = w.inputs(seed=100 + rank, device=dev)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)

    def step():
        lat = runner.sample_with_context(inp["vox"], inp["context"], noise=inp["noise"])
        if dist is not None:
            vd.gather_latents([lat], rank, ws)
        return lat

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if args.profile:
        torch.cuda.nvtx.range_push("profile_step")
        step()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        print(json.dumps({"profile_step": "done", "launches": _lib.launch_count()}))
        return

    # ---------------------------------------------------------------- timed region (device time)
    s = torch.cuda.current_stream()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    launches0 = _lib.launch_count()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    ktimer: dict = {}
    # inside the timed steps only the dominant kernel (window self-attention) is bracketed by
    # CUDA events; the other ~1700 launches of a sample run without them
    runner.kernel_timer = ktimer
    runner.kernel_timer_kinds = {"attention_window_self"}
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            _l2_flush(flush)
            evs[i][0].record(s)
            step()
            evs[i][1].record(s)
        torch.cuda.synchronize()
    runner.kernel_timer = None
    runner.kernel_timer_kinds = None
    launches = (_lib.launch_count() - launches0) // max(args.steps, 1)
    # every kernel class of the forward, in one more sample after the timed steps (not timed
    # as a step): CUDA events around each launch on its stream
    kstep: dict = {}
    _l2_flush(flush)
    runner.kernel_timer = kstep
    step()
    torch.cuda.synchronize()
    runner.kernel_timer = None
    total_ms = sum(a.elapsed_time(b) for a, b in evs)
    t = torch.tensor([total_ms], device=dev)
    if dist is not None:
        dist.barrier()
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_step = float(t.item()) / args.steps
    value = ws * NFE_PER_SAMPLE * w.n / (ms_step / 1e3)

    # ---------------------------------------------------------------- per-branch NFE times
    geom = runner._prepare_sample_geometry([inp["vox"]], inp["context"])
    xs = inp["noise"][geom["perm"]].contiguous()
    nfe = {}
    for name, kw in (("pos", {}), ("neg_1tok", {"uncond": True})):
        if name == "neg_1tok":
            runner._b0_share = None
        runner.forward_flow_fast(xs, 0.9, inp["context"], None, geom, **kw)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(s)
        for _ in range(3):
            if name == "neg_1tok":
                runner._b0_share = None
            runner.forward_flow_fast(xs, 0.9, inp["context"], None, geom, **kw)
        e1.record(s)
        torch.cuda.synchronize()
        nfe[name] = {"ms": e0.elapsed_time(e1) / 3, "voxel_tokens_per_s": w.n / (e0.elapsed_time(e1) / 3e3)}
    # the kernel classes of one NFE of each branch with every kernel alone on the GPU: one NFE at
    # a time and its context-stream work on the voxel stream (no overlap inside the NFE either)
    ksolo: dict = {}
    overlap = runner.overlap_context
    runner.overlap_context = False
    for name, kw in (("pos", {}), ("neg_1tok", {"uncond": True})):
        if name == "neg_1tok":
            runner._b0_share = None
        _l2_flush(flush)
        runner.kernel_timer = ksolo
        runner.forward_flow_fast(xs, 0.9, inp["context"], None, geom, **kw)
        runner.kernel_timer = None
    torch.cuda.synchronize()
    runner.overlap_context = overlap

    # ---------------------------------------------------------------- e2e through the plugin API
    vox_h = inp["vox_host"].pin_memory()
    dino_h = inp["dino_host"].pin_memory()
    cond = LatDitConditioning(dino_features=dino_h, batch_size=1)
    gen = torch.Generator(device=dev).manual_seed(7)
    sol.generate([vox_h], conditioning=cond, generator=gen)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    e2e_ms = []
    for _ in range(args.steps):
        _l2_flush(flush)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        lat = sol.generate([vox_h], conditioning=cond, generator=gen)[0]
        lat_h = lat.cpu()
        if dist is not None:
            vd.gather_latents([lat], rank, ws)
        torch.cuda.synchronize()
        e2e_ms.append((time.perf_counter() - t0) * 1e3)
    te = torch.tensor([statistics.median(e2e_ms)], device=dev)
    if dist is not None:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = ws * NFE_PER_SAMPLE * w.n / (float(te.item()) / 1e3)
    h2d = vox_h.numel() * vox_h.element_size() + dino_h.numel() * dino_h.element_size()
    d2h = lat_h.numel() * lat_h.element_size()

    # ---------------------------------------------------------------- roofline of the attention kernel
    hbm, tflops_peak, peak_kind = _peaks()
    tflops_sustained = _peaks_sustained()
    # live: average duration of the window self-attention launches inside the timed steps
    # (CUDA events on their stream), against the sustained GEMM peak
    att_events = ktimer["attention_window_self"]
    live_ms = statistics.fmean(a.elapsed_time(b) for a, b, _, _ in att_events)
    flops = statistics.fmean(u for _, _, u, _ in att_events)
    achieved = flops / (live_ms / 1e3) / 1e12
    # the same launches restricted to steps where only one NFE runs (the unguided step):
    # in guided steps the conditional and the 1-token NFE run on two streams and share the GPU
    solo = [(a, b) for a, b, _, shared in att_events if not shared]
    solo_ms = statistics.fmean(a.elapsed_time(b) for a, b in solo) if solo else None
    flops_alone, att_ms_alone = attention_roofline(w, runner)
    traffic = attention_traffic()
    kernels = kernel_table(kstep, hbm, tflops_sustained, peak_kind, solo=ksolo)
    assert _lib.device_error() == 0, "device error word set during the benchmark"

    # ---------------------------------------------------------------- C5 sharded batch (strong scaling)
    c5 = None
    if not args.no_c5:
        del sol, runner
        torch.cuda.empty_cache()
        c5 = c5_bench(rank, ws, dev, dist, steps=args.c5_steps, warmup=1, model=model)

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        v, dt = cpu_baseline_sample(threads)
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{CPU_SAMPLE} ({dt:.1f} s)"}

    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded shell voxels, N(0,1) context, "
                                                          "random-init weights)",
            "config": {"workload": "C4 full 24-block DiT: dim 1536, 12x128 heads, N=16384 shell r=36 in 64^3, "
                                   "4101x1536 context, 4-step exact solver (3 guided CFG 3.0 + 1) = 7 NFE",
                       "global_batch": ws, "seq_len": w.n, "parallelism": f"samples x{ws}",
                       "l2": "256 MiB L2 flush before every timed step; 3.9 GB of weights streamed per NFE"},
            "nfe": nfe,
            "generate_latency_ms": float(te.item()),
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "api": "Solution.generate (pinned host voxels + fp16 DINO in, latents to host)"},
            "gpu_launches": int(launches),
            "roofline": {"kernel": "attention_kernel<128> (window self-attention, 4x4096 voxels, 12x128)",
                         "bound": "tensor", "achieved": achieved, "peak": tflops_sustained, "unit": "TFLOP/s",
                         "frac": achieved / tflops_sustained,
                         "peak_kind": f"{peak_kind} sustained bf16 (kernel timed inside the timed steps)",
                         "flops_per_launch": flops, "ms_per_launch": live_ms, "launches": len(att_events),
                         "traffic": traffic,
                         "traffic_source": "dram__bytes_read.sum + dram__bytes_write.sum of one ncu capture of "
                                           "the same kernel source (profiles/attention_traffic.json)",
                         "kernels": kernels,
                         "kernels_source": "one sample run right after the timed steps with CUDA events around "
                                           "every launch (the timed steps carry events around the window "
                                           "self-attention launches only)",
                         "unshared": None if solo_ms is None else {
                             "ms_per_launch": solo_ms, "launches": len(solo),
                             "achieved": flops / (solo_ms / 1e3) / 1e12,
                             "frac": flops / (solo_ms / 1e3) / 1e12 / tflops_sustained,
                             "note": "launches of the unguided step, where no second NFE shares the GPU"},
                         "alone": {"ms_per_launch": att_ms_alone,
                                   "achieved": flops_alone / (att_ms_alone / 1e3) / 1e12,
                                   "peak": tflops_peak, "peak_kind": f"{peak_kind} burst bf16",
                                   "frac": flops_alone / (att_ms_alone / 1e3) / 1e12 / tflops_peak}},
            "cpu_baseline": cpu,
            "clocks": clk.summary(),
            "c5": c5,
        }), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
