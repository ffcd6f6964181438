"""The packed-weight directory on the GPU: write_packed produces the reference's bytes (pack_b of each B operand,
bit-exact against the oracle) and a manifest that read_manifest verifies; a DiT loaded from the directory
(load_packed) gives the same velocity, bit for bit, as one built from the float weights."""

import numpy as np
import pytest

from oracle import bfp16_oracle as O

pytestmark = pytest.mark.gpu


def test_write_load_roundtrip(tmp_path):
    import torch
    from redline_tiny_b200 import dit, ops, weights as W
    cfg = dit.DiTConfig(hidden=256, heads=2, ffn=512, blocks=2, text=64, image=192, grid=(12, 16))
    w = dit.random_weights(cfg, seed=11)
    man = W.write_packed(tmp_path, w, cfg)
    assert set(man["blocks"]) == {"00", "01"}
    raw = W.read_manifest(tmp_path)                                   # sizes and sha256 verified
    b1 = w["blocks"][1]
    assert np.array_equal(raw["blocks"][1]["qkv"], O.pack_b(b1["qkv"].cpu().numpy()))
    assert np.array_equal(raw["blocks"][1]["up"],
                          O.pack_b(dit.interleave_up_torch(b1["gate"], b1["proj"]).cpu().numpy()))
    pad = np.zeros((cfg.hidden, 1024), np.float32)
    pad[:, :128] = w["proj_out"].cpu().numpy()
    assert np.array_equal(raw["proj_out"], O.pack_b(pad))

    loaded = W.load_packed(tmp_path)
    rng = np.random.default_rng(4)
    lat = torch.from_numpy(rng.standard_normal((cfg.image, cfg.latent_ch)).astype(np.float32))
    txt = torch.from_numpy(rng.standard_normal((cfg.text, cfg.hidden)).astype(np.float32))
    v_packed = dit.DiT(cfg, loaded).forward(lat, txt, 0.5).float().cpu()
    v_float = dit.DiT(cfg, w).forward(lat, txt, 0.5).float().cpu()
    ops.device_status()
    assert torch.equal(v_packed, v_float)
