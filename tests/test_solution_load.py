"""The plugin's load path on CPU: weight discovery in the reference's order
(``solution.py:48-102``) and the folding of a distilled adapter into the weights
(``solution.py:105-132``).  Where ``VDIT_REFERENCE_DIR`` names a reference checkout,
the reference's own folding function runs on the same synthetic adapter too."""
import importlib.util
import os

import pytest
import torch

from vdit.solution import _discover_weights_dir, merge_distilled_adapters

from oracle import reference_root


def _weights(d):
    d.mkdir(parents=True, exist_ok=True)
    (d / "diffusion_pytorch_model.safetensors").write_bytes(b"")
    return d


def test_discovery_order(tmp_path, monkeypatch):
    primary = tmp_path / "submission"
    primary.mkdir()
    a = _weights(tmp_path / "a" / "lat_dit")
    vae = tmp_path / "b" / "lat_vae"
    vae.mkdir(parents=True)
    b = _weights(tmp_path / "b" / "lat_dit")
    e = _weights(tmp_path / "env")
    monkeypatch.chdir(tmp_path)
    # nothing anywhere: the primary path
    assert _discover_weights_dir(primary, argv=[], environ={}) == primary
    # --lat-dit-dir X (X/lat_dit holds the weights) and the = form
    assert _discover_weights_dir(primary, argv=["x", "--lat-dit-dir", str(tmp_path / "a")], environ={}) == a
    assert _discover_weights_dir(primary, argv=[f"--lat-dit-dir={a}"], environ={}) == a
    # --lat-vae-dir X: the lat_dit directory beside X, both forms
    assert _discover_weights_dir(primary, argv=["--lat-vae-dir", str(vae)], environ={}) == b
    assert _discover_weights_dir(primary, argv=[f"--lat-vae-dir={vae}"], environ={}) == b
    # the first matching argument wins, before any environment variable
    assert _discover_weights_dir(primary, argv=["--lat-vae-dir", str(vae), "--lat-dit-dir", str(a)],
                                 environ={"LAT_DIT_DIR": str(e)}) == b
    # environment variables in order
    assert _discover_weights_dir(primary, argv=[], environ={"KANDI3D_WEIGHTS_DIR": str(e)}) == e
    assert _discover_weights_dir(primary, argv=[], environ={"LAT_DIT_WEIGHTS_DIR": str(tmp_path / "a"),
                                                            "KANDI3D_WEIGHTS_DIR": str(e)}) == a
    # organiser location relative to the working directory
    w = _weights(tmp_path / "weights" / "lat_dit")
    assert _discover_weights_dir(primary, argv=[], environ={}) == w.resolve()
    # the primary path and its lat_dit beat everything
    p2 = _weights(primary / "lat_dit")
    assert _discover_weights_dir(primary, argv=["--lat-dit-dir", str(a)], environ={"LAT_DIT_DIR": str(e)}) == p2


def _state():
    g = torch.Generator().manual_seed(3)
    return {"flow.blocks.0.to_qkv.weight": torch.randn(12, 8, generator=g),
            "flow.blocks.0.to_out.weight": torch.randn(8, 8, generator=g).to(torch.bfloat16),
            "flow.blocks.0.ffn_conv.weight": torch.randn(3, 3, 3, 16, generator=g),
            "image_map.bias": torch.randn(8, generator=g)}


def _adapter():
    g = torch.Generator().manual_seed(4)
    return {"lora_scale": 0.5,
            "lora_A": {"flow.blocks.0.to_qkv.weight": torch.randn(4, 8, generator=g),
                       "flow.blocks.0.to_out.weight": torch.randn(2, 8, generator=g),
                       "flow.blocks.9.to_out.weight": torch.randn(2, 8, generator=g),      # not in the model
                       "flow.blocks.0.ffn0.weight": torch.randn(2, 8, generator=g)},       # no B: skipped
            "lora_B": {"flow.blocks.0.to_qkv.weight": torch.randn(12, 4, generator=g),
                       "flow.blocks.0.to_out.weight": torch.randn(8, 2, generator=g).to(torch.bfloat16),
                       "flow.blocks.9.to_out.weight": torch.randn(8, 2, generator=g)},
            "weight_deltas": {"flow.blocks.0.ffn_conv.weight": 1e-3 * torch.randn(3, 3, 3, 16, generator=g),
                              "flow.blocks.0.to_qkv.weight": 1e-2 * torch.randn(12, 8, generator=g),
                              "missing.weight": torch.randn(3, generator=g)}}


def test_merge_distilled_adapters(tmp_path):
    state, ad = _state(), _adapter()
    torch.save(ad, tmp_path / "student_adapter.pt")
    want = {k: v.float().clone() for k, v in state.items()}
    s = ad["lora_scale"]
    for k in ("flow.blocks.0.to_qkv.weight", "flow.blocks.0.to_out.weight"):
        want[k] = want[k] + (ad["lora_B"][k].float() @ ad["lora_A"][k].float()) * s
    for k in ("flow.blocks.0.ffn_conv.weight", "flow.blocks.0.to_qkv.weight"):
        want[k] = want[k] + ad["weight_deltas"][k]
    assert merge_distilled_adapters(state, tmp_path) == 4
    for k in want:
        assert state[k].dtype == torch.float32
        assert torch.equal(state[k], want[k]), k
    assert set(state) == set(want)


def test_merge_without_or_with_unreadable_adapter(tmp_path):
    state = _state()
    before = {k: v.clone() for k, v in state.items()}
    assert merge_distilled_adapters(state, tmp_path) == 0
    (tmp_path / "student_adapter.pt").write_bytes(b"not a torch file")
    assert merge_distilled_adapters(state, tmp_path) == 0
    for k in before:
        assert torch.equal(state[k], before[k])


@pytest.mark.skipif(reference_root() is None, reason="VDIT_REFERENCE_DIR does not name a reference checkout")
def test_merge_matches_reference_function(tmp_path):
    """The reference's ``_merge_distilled_adapters_if_present`` on fp32 parameters (its model
    is fp32) against ours on the same checkpoint tensors: identical results."""
    from tests.golden.make_golden import load_reference
    ref = reference_root()
    os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
    load_reference(ref)
    spec = importlib.util.spec_from_file_location("ref_solution_module", ref / "solution.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    torch.save(_adapter(), tmp_path / "student_adapter.pt")
    params = {k: v.float().clone() for k, v in _state().items()}

    class Core:
        def state_dict(self):
            return params

    class Model:
        core = Core()

    mod._merge_distilled_adapters_if_present(Model(), tmp_path)
    ours = _state()
    merge_distilled_adapters(ours, tmp_path)
    for k in params:
        assert torch.equal(ours[k], params[k]), k
