"""The on-disk sample format (voxel indices + cached DINOv3 features) on CPU: the lookup
order of the reference's evaluation driver, shapes and dtypes handed to the plugin, and
the reference's own public-test samples read in place where its checkout is present."""
from pathlib import Path

import numpy as np
import pytest
import torch

from vdit import ingest

from oracle import reference_root

_REF = reference_root()
REF_SAMPLES = _REF / "fetched_info" / "sample_test_data" / "public_test" if _REF else Path("/nonexistent")


def _write_sample(root: Path, sid: str, n: int, view: str = "4view_000", key: str = "vox_idxi", cache=True):
    d = root / sid / "cache" if cache else root / sid
    d.mkdir(parents=True)
    rng = np.random.default_rng(n)
    vox = rng.integers(0, 64, size=(n, 3)).astype(np.int32)
    np.savez(d / "vox_idxi.npz", **{key: vox})
    feats = rng.standard_normal((1, 4101, 1280)).astype(np.float16)
    token = rng.standard_normal((1, 1280)).astype(np.float16)
    np.savez(d / (f"{view}_dinov3.npz" if view else "dinov3.npz"), feats=feats, token=token)
    return vox, feats, token


def test_load_sample_shapes_and_values(tmp_path):
    vox, feats, token = _write_sample(tmp_path, "a", 100)
    vl, cond = ingest.load_sample(tmp_path / "a")
    assert len(vl) == 1 and vl[0].dtype == torch.int32 and vl[0].shape == (100, 3)
    assert np.array_equal(vl[0].numpy(), vox)
    assert cond.dino_features.shape == (1, 4101, 1280) and cond.dino_features.dtype == torch.float16
    assert np.array_equal(cond.dino_features.numpy(), feats) and np.array_equal(cond.dino_token.numpy(), token)
    assert cond.batch_size == 1


def test_lookup_order_and_fallbacks(tmp_path):
    _write_sample(tmp_path, "b", 10, view="", key="arr_0", cache=False)     # dinov3.npz, arr_0, no cache/
    vl, cond = ingest.load_sample(tmp_path / "b")
    assert vl[0].shape == (10, 3) and cond.dino_features.shape[1] == 4101
    d = tmp_path / "c"
    d.mkdir()
    np.savez(d / "vox_idxi.npz", vox_idxi=np.zeros((3, 3), np.int32))
    torch.save(torch.ones(1, 4101, 1280, dtype=torch.float16), d / "dinov3_feats.pt")
    torch.save(torch.ones(1, 1280, dtype=torch.float16), d / "dinov3_token.pt")
    _, cond = ingest.load_sample(d)
    assert float(cond.dino_features.float().mean()) == 1.0
    assert ingest.list_samples(tmp_path) == ["b", "c"]
    e = tmp_path / "e"
    e.mkdir()
    np.savez(e / "vox_idxi.npz", vox_idxi=np.zeros((3, 3), np.int32))
    with pytest.raises(FileNotFoundError):                        # no features for the view
        ingest.load_sample(e)
    np.savez(e / "bad.npz", vox_idxi=np.zeros((3, 4), np.int32))
    with pytest.raises(ValueError, match=r"\[N, 3\]"):
        ingest.load_vox_idxi(e / "bad.npz")


@pytest.mark.skipif(not REF_SAMPLES.is_dir(), reason="VDIT_REFERENCE_DIR does not name a reference checkout")
def test_reference_public_samples_in_place():
    ids = ingest.list_samples(REF_SAMPLES)
    assert ids, "no public-test sample with 4view_000 features"
    vl, cond = ingest.load_sample(REF_SAMPLES / ids[0])
    assert vl[0].dtype == torch.int32 and vl[0].shape[1] == 3 and 4000 < vl[0].shape[0] < 7000
    assert cond.dino_features.shape == (1, 4101, 1280) and cond.dino_features.dtype == torch.float16
    assert cond.dino_token.shape == (1, 1280)
