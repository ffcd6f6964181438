"""The packed-weight directory reader (redline_tiny_b200.weights.read_manifest) on a directory laid out as the
reference's pack_weights.py writes it (manifest.json with per-file sizes and sha256, bNN_*.bin = pack_b bytes,
norm .npy files, host/*.npy), built here with the oracle's pack_b. Host-only: no GPU."""

import hashlib
import json

import numpy as np
import pytest

from oracle import bfp16_oracle as O
from redline_tiny_b200 import weights as W


def _entry(path, raw, K, N):
    return {"file": path.name, "K": K, "N": N, "bytes": int(raw.size), "sha256": hashlib.sha256(raw).hexdigest(),
            "source": ["test"], "B": "test"}


@pytest.fixture
def packed_dir(tmp_path):
    rng = np.random.default_rng(3)
    D, F = 128, 256
    man = {"layout": {"format": "bfp16ebs8"}, "blocks": {}, "host": {}}
    mats = {}
    for name, (K, N) in (("img_in", (64, D)), ("proj_out", (D, 1024))):
        B = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
        raw = O.pack_b(B)
        raw.tofile(tmp_path / f"{name}.bin")
        man[name] = _entry(tmp_path / f"{name}.bin", raw, K, N)
        mats[name] = raw
    for i in range(2):
        e = {}
        for name, (K, N) in (("qkv", (D, 3 * D)), ("o", (D, D)), ("up", (D, 2 * F)), ("down", (F, D))):
            raw = O.pack_b((rng.standard_normal((K, N)) * 0.02).astype(np.float32))
            path = tmp_path / f"b{i:02d}_{name}.bin"
            raw.tofile(path)
            e[name] = _entry(path, raw, K, N)
            mats[i, name] = raw
        for name in ("norm_q", "norm_k"):
            np.save(tmp_path / f"b{i:02d}_{name}.npy", np.ones(128, np.float32))
            e[name] = {"file": f"b{i:02d}_{name}.npy", "shape": [128], "dtype": "float32"}
        man["blocks"][f"{i:02d}"] = e
    (tmp_path / "host").mkdir()
    np.save(tmp_path / "host" / "modulation.1.weight.npy", np.arange(6, dtype=np.float32).reshape(2, 3))
    man["host"]["modulation.1.weight"] = {"file": "host/modulation.1.weight.npy", "shape": [2, 3], "dtype": "float32"}
    (tmp_path / "manifest.json").write_text(json.dumps(man, indent=1))
    return tmp_path, mats


def test_reads_every_file(packed_dir):
    d, mats = packed_dir
    got = W.read_manifest(d)
    assert np.array_equal(got["img_in"], mats["img_in"]) and np.array_equal(got["proj_out"], mats["proj_out"])
    assert len(got["blocks"]) == 2
    for i in range(2):
        for name in W.BIN_NAMES:
            assert np.array_equal(got["blocks"][i][name], mats[i, name])
        assert got["blocks"][i]["norm_q"].shape == (128,)
    assert np.array_equal(got["host"]["modulation.1.weight"], np.arange(6, dtype=np.float32).reshape(2, 3))
    assert len(W.read_manifest(d, blocks=[1])["blocks"]) == 1


def test_rejects_a_corrupt_file(packed_dir):
    d, _ = packed_dir
    raw = np.fromfile(d / "b01_up.bin", np.uint8)
    raw[1000] ^= 1
    raw.tofile(d / "b01_up.bin")
    with pytest.raises(ValueError, match="sha256"):
        W.read_manifest(d)
    W.read_manifest(d, verify=False)       # the check can be skipped, as the reference's loader does


def test_rejects_a_short_or_missing_file(packed_dir):
    d, _ = packed_dir
    raw = np.fromfile(d / "b00_o.bin", np.uint8)
    raw[:-9].tofile(d / "b00_o.bin")
    with pytest.raises(ValueError, match="bytes"):
        W.read_manifest(d, verify=False)
    (d / "b00_o.bin").unlink()
    with pytest.raises(ValueError, match="missing"):
        W.read_manifest(d)
