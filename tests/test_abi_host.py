"""CPU tests: the C-ABI library loads and exports every declared symbol, and
the host-side logic (schedule, solver config, plugin contract, window
partition, architecture/keys) matches the oracle/reference behaviour."""
import json
import re
from pathlib import Path

import numpy as np
import pytest
import torch

import vdit
from vdit import _lib
from vdit import fast_kernels as fk
from vdit.fast_sampler import SolverConfig, build_schedule
from vdit.model import LatDitArch, param_shapes
from vdit.runtime import FlowMatchSamplingParams, LatDitGenerator, resolve

from oracle import geometry as geo
from oracle import model as om

ROOT = Path(__file__).resolve().parents[1]


def _declared():
    text = (ROOT / "include" / "vdit.h").read_text()
    return sorted(set(re.findall(r"\b(vdit_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = _declared()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_lib.SIGNATURES), set(names) ^ set(_lib.SIGNATURES)


def test_error_strings_and_host_queries():
    lib = _lib.load()
    assert b"sm_100a" in lib.vdit_version()
    for code in (0, -1, -2, -3, -4, -5, -6):
        assert lib.vdit_error_string(code)
    assert lib.vdit_launch_count() >= 0
    assert lib.vdit_attention_1q_workspace_bytes(12, 128, 16384) > 0
    assert lib.vdit_attention_1q_workspace_bytes(0, 128, 16384) == 0


def test_shape_errors_are_reported_before_any_launch():
    lib = _lib.load()
    # null pointers / bad shapes are rejected on the host (no GPU needed)
    assert lib.vdit_modulate(None, 10, 1536, None, None, None, None) == -1
    assert lib.vdit_attention(None, 0, None, 0, None, 0, None, 0, None, None, None, 0, 12, 128, 1.0, None) == -1
    assert lib.vdit_dwconv27(None, 5, 7680, None, None, None, None, 1, None) == -1
    assert lib.vdit_dwconv27_plan_bytes(0) == 0
    assert lib.vdit_dwconv27_plan_bytes(129) == 2 * lib.vdit_dwconv27_plan_bytes(128)
    assert lib.vdit_dwconv27_plan(None, None, 5, None, 0, None) == -1
    assert lib.vdit_dwconv27_plan(16, 16, 5, 16, 0, None) == -5            # plan buffer too small
    assert lib.vdit_dwconv27_swiglu_planned(None, 5, 7680, None, None, None, None, None) == -1
    assert lib.vdit_dwconv27_swiglu_planned(16, 5, 960, 16, 16, 16, 16, None) == -4   # c % 128 != 0
    assert lib.vdit_dwconv27_swiglu_planned_bf16w(None, 5, 7680, None, None, None, None, None) == -1
    assert lib.vdit_dwconv27_swiglu_planned_bf16w(16, 5, 960, 16, 16, 16, 16, None) == -4
    assert lib.vdit_unpatchify_project(None, 10, 1536, None, None, None) == -1
    assert lib.vdit_unpatchify_project(16, 10, 1540, 16, 16, None) == -1           # d % 8 != 0
    assert lib.vdit_unpatchify_project(8, 10, 1536, 16, 16, None) == -2            # y not 16-byte aligned
    assert lib.vdit_unpatchify_project(16, 0, 1536, 16, 16, None) == 0             # nothing to do
    assert lib.vdit_split_weight3(None, 16, 1536, None, None) == -1
    with pytest.raises(RuntimeError, match="invalid argument"):
        _lib.check(-1, "probe")


def test_rope2d_tables_must_cover_the_context():
    qkv = torch.zeros(5 + 10, 3 * 256, dtype=torch.bfloat16)
    cos, sin = torch.zeros(9, 2, 32), torch.zeros(9, 2, 32)         # a 3x3 grid: 9 of the 10 tokens
    with pytest.raises(ValueError, match="RoPE tables"):
        fk.fused_qknorm_rope2d_cond_inplace(qkv, torch.ones(256), torch.ones(256), cos, sin, 2, 128)


def test_attention_offsets_must_stay_inside_the_tensors():
    q = torch.zeros(100, 256, dtype=torch.bfloat16)
    kv = torch.zeros(60, 512, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="past q/k/v"):
        fk.attention(q, kv[:, :256], kv[:, 256:], [0, 50, 100], [0, 30, 61], 2, 128)
    with pytest.raises(ValueError, match="out_rows"):
        fk.attention(q, kv[:, :256], kv[:, 256:], [0, 100], [0, 60], 2, 128,
                     out_rows=torch.arange(99))
    with pytest.raises(ValueError, match="same number"):
        fk.attention(q, kv[:, :256], kv[:, 256:], [0, 100], [0, 30, 60], 2, 128)
    with pytest.raises(ValueError, match="run past"):
        fk.attention_1q(torch.zeros(256, dtype=torch.bfloat16), kv, 2, 128, k_offset=256)


def test_voxel_coordinates_must_be_n_by_3():
    from vdit import fast_kernels as fk
    for bad in (torch.zeros(10, 4, dtype=torch.int32), torch.zeros(10, dtype=torch.int32)):
        with pytest.raises(ValueError, match=r"\[N, 3\]"):
            fk.lex_perm(bad)


@pytest.mark.parametrize("steps,guided", [(4, 3), (8, 6), (14, None)])
def test_build_schedule_matches_oracle(steps, guided):
    cfg = SolverConfig(num_inference_steps=steps, n_guided_steps=guided or 10,
                       n_unguided_steps=(steps - guided) if guided else 4)
    t, g, ng = build_schedule(cfg)
    if guided:
        to, go = om.build_schedule(steps, guided, 3.0, (0.5, 1.0))
        assert torch.allclose(t, to) and g == go and ng == guided
    assert t[0] == 1.0 and t[-1] == 0.0 and len(g) == steps


def test_solver_config_reads_json_and_ignores_approximations(tmp_path):
    (tmp_path / "solver_config.json").write_text(json.dumps(
        {"num_inference_steps": 4, "guidance_scale": 3.0, "qaoa_enabled": True, "solver_type": "piecewise_qaoa",
         "cfg_stride": 2, "unknown_key": 1}))
    cfg = SolverConfig.from_dir(tmp_path, fallback_model_cfg={"cfg": 7.0, "rescale_t": 3.0})
    assert cfg.guidance_scale == 3.0 and cfg.solver_type == "piecewise_euler" and cfg.cfg_stride == 1
    assert "qaoa_enabled" in cfg.approximate_fields_ignored


def test_solver_config_approximate_cfg_cache_is_opt_in(tmp_path):
    """A config asking for the reference's CFG cache ("neg_reuse", stride 2, unconditional NFE at
    guided steps 0 and 2) keeps the exact solver unless the caller opts in."""
    (tmp_path / "solver_config.json").write_text(json.dumps(
        {"cfg_cache_mode": "neg_reuse", "cfg_stride": 2, "eval_uncond_steps": [0, 2], "qaoa_enabled": True}))
    exact = SolverConfig.from_dir(tmp_path)
    assert not exact.approximate_cfg_cache and exact.cfg_stride == 1 and exact.eval_uncond_steps == []
    assert {"cfg_cache_mode=neg_reuse", "cfg_stride=2", "eval_uncond_steps=[0, 2]"} <= set(exact.approximate_fields_ignored)
    approx = SolverConfig.from_dir(tmp_path, allow_approximate_cfg_cache=True)
    assert approx.approximate_cfg_cache and approx.cfg_stride == 2 and approx.eval_uncond_steps == [0, 2]
    assert "qaoa_enabled" in approx.approximate_fields_ignored          # the QAOA solver is never taken
    on = SolverConfig().enable_approximate_cfg_cache()
    assert on.approximate_cfg_cache and on.eval_uncond_steps == [0, 2] and on.cfg_zero_star_projection


def test_runtime_merge_and_generator_contract():
    base = FlowMatchSamplingParams(guidance_scale=7.0, num_inference_steps=4)
    r = resolve(base, FlowMatchSamplingParams(guidance_scale=3.0), cfg_range=[0.4, 1.0])
    assert r.guidance_scale == 3.0 and r.cfg_range == (0.4, 1.0)
    with pytest.raises(TypeError):
        class Bad(LatDitGenerator):  # noqa: F811
            def generate(self, *a, **k):
                return None


@pytest.mark.parametrize("n", [1, 4095, 4096, 4097, 16384, 70000])
def test_window_partition_matches_oracle(n):
    cu, mx = fk.window_seqlens([n], 4096)
    assert np.array_equal(np.array(cu), geo.window_cu_seqlens(n, 4096))
    assert mx == min(n, 4096)


def test_param_keys_match_oracle_and_checkpoint_names():
    a = LatDitArch(dim=192, head_dim=96, depth=3, cond_depth=1)
    o = om.ModelConfig(dim=192, head_dim=96, depth=3, cond_depth=1)
    assert param_shapes(a) == om.param_shapes(o)
    full = param_shapes(LatDitArch())
    assert full["flow.blocks.0.ffn_conv.weight"] == (3, 3, 3, 7680)
    assert full["flow.blocks.8.cond_gates.weight"] == (3072, 1536)
    assert full["flow.blocks.0.qk_norm.q_scale"] == (16, 96)


def test_arch_rejects_unbuilt_variants():
    with pytest.raises(NotImplementedError):
        LatDitArch.from_model_config({"io_conv": True})
    a = LatDitArch.from_model_config({"dim": 1536, "head_dim": 96})
    assert a.heads == 16


def test_weights_are_bf16_detects_bf16_values():
    """The check that selects the bf16-operand conv: true exactly when every fp32 value
    is a bf16 value (a bf16 model upcast), on any device."""
    g = torch.Generator().manual_seed(0)
    w = torch.randn(27, 256, generator=g)
    assert not fk.weights_are_bf16(w)
    wb = w.to(torch.bfloat16).float()
    assert fk.weights_are_bf16(wb)
    wb[3, 7] = wb[3, 7].nextafter(torch.tensor(float("inf")))   # one value off the bf16 grid
    assert not fk.weights_are_bf16(wb)
    assert fk.weights_are_bf16(torch.zeros(27, 8)) and fk.weights_are_bf16(torch.full((4,), -2.0 ** -130))


def _c_kind(param: str) -> str:
    """'ptr', 'int' or 'float' for one C parameter declaration of include/vdit.h."""
    p = param.strip()
    if "*" in p or p.startswith("vdit_stream_t"):
        return "ptr"
    if p.startswith(("float", "double")):
        return "float"
    return "int"


def _py_kind(t) -> str:
    import ctypes
    if t in (ctypes.c_void_p, ctypes.c_char_p):
        return "ptr"
    if t in (ctypes.c_float, ctypes.c_double):
        return "float"
    return "int"


def test_ctypes_signatures_match_the_header():
    """Every binding in _lib.SIGNATURES passes as many arguments, of the same kind (pointer,
    integer, floating point) and in the same order, as its declaration in include/vdit.h."""
    text = re.sub(r"/\*.*?\*/", " ", (ROOT / "include" / "vdit.h").read_text(), flags=re.S)
    decls = dict(re.findall(r"\b(vdit_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text))
    assert set(decls) == set(_lib.SIGNATURES)
    for name, params in decls.items():
        c = [] if params.strip() in ("", "void") else [_c_kind(x) for x in params.split(",")]
        py = [_py_kind(t) for t in _lib.SIGNATURES[name][1]]
        assert c == py, f"{name}: header {c} vs ctypes {py}"
