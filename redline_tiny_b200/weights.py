"""The reference's packed-weight directory, written and read on a B200.

Layout (redline/pack_weights.py:1-17, 92-118, 129-182):

    manifest.json          {"layout": ..., "img_in": entry, "proj_out": entry, "blocks": {"NN": {name: entry}},
                            "host": {tensor: {"file", "shape", "dtype"}}, "total_block_bytes": ...}
                           a .bin entry is {"file", "K", "N", "bytes", "sha256", "source", ...}
    bNN_qkv.bin            B = [Wq^T | Wk^T | Wv^T]               (K = hidden, N = 3 hidden)
    bNN_o.bin              B = Wo^T                               (hidden, hidden)
    bNN_up.bin             B = [gate 64 | proj 64] per 128 columns (hidden, 2 FFN)
    bNN_down.bin           B = Wdown^T                            (FFN, hidden)
    bNN_norm_q.npy, bNN_norm_k.npy   float32 (128,)
    img_in.bin             B = W^T (latent channels, hidden)
    proj_out.bin           B = W^T zero-padded to 1024 output columns (hidden, 1024)
    host/<tensor>.npy      every non-block tensor, float32

Each .bin holds the raw bytes of to_bfp16(b_layout(B, 64, 128)) (pack_weights.pack_b), 9 bytes per 8 weights.

write_packed(directory, weights, cfg)     packs every B on the GPU (rl_pack_b) and writes files + manifest.
read_manifest(directory, blocks, verify)  host side: the manifest and the raw bytes, each .bin checked against the
                                          manifest's size and sha256 (ValueError on a mismatch or a missing file),
                                          as the reference's prepare.py verification does (prepare.py:95-115).
load_packed(directory, cfg, ...)          read_manifest + the device upload and the one-time conversion to the
                                          native tile format, giving the weight dict `dit.DiT` takes - the
                                          resident `Weights` of forward.py:175-191.
"""

import hashlib
import json
from pathlib import Path

import numpy as np
import torch

from . import ops

BIN_NAMES = ("qkv", "o", "up", "down")
NORM_NAMES = ("norm_q", "norm_k")
PROJ_OUT_COLS = 1024    # the reference pads proj_out to its program's 1024 output columns


def _sha256(raw):
    return hashlib.sha256(memoryview(np.ascontiguousarray(raw, dtype=np.uint8))).hexdigest()


def _bin_entry(path, raw, K, N, how):
    return {"file": path.name, "K": int(K), "N": int(N), "bytes": int(raw.size), "sha256": _sha256(raw), "B": how}


def write_packed(directory, weights, cfg):
    """Write `weights` (the float layout of dit.random_weights: B operands as (K, N) tensors) in the reference's
    packed format. Returns the manifest dict."""
    from .dit import interleave_up_torch
    out = Path(directory)
    out.mkdir(parents=True, exist_ok=True)
    (out / "host").mkdir(exist_ok=True)

    def pack(B):
        B = B if B.is_cuda else B.cuda()
        return ops.pack_b(B.float().contiguous()).cpu().numpy()

    man = {
        "model": "redline-tiny DiT (B200 packer)",
        "config": {"hidden": cfg.hidden, "heads": cfg.heads, "ffn": cfg.ffn, "blocks": cfg.blocks,
                   "latent_ch": cfg.latent_ch, "temb_dim": cfg.temb_dim},
        "layout": {"format": "bfp16ebs8, 9 bytes per 8 values ([shared exp][8 x int8]), round half to even",
                   "B": "b_layout(B, k=64, n=128) of B = K x N (C = A @ B)",
                   "up_columns": "per 128-col tile: [gate 64 | proj 64]"},
    }
    host = {}
    for name, a in weights["host"].items():
        a = np.asarray(a, np.float32)
        np.save(out / "host" / f"{name}.npy", a)
        host[name] = {"file": f"host/{name}.npy", "shape": list(a.shape), "dtype": "float32"}
    man["host"] = host
    proj = weights["proj_out"]
    padded = torch.zeros(proj.shape[0], PROJ_OUT_COLS, dtype=torch.float32, device=proj.device)
    padded[:, :proj.shape[1]] = proj
    for name, B, how in (("img_in", weights["img_in"], "W^T"), ("proj_out", padded, "W^T zero-padded to 1024")):
        raw = pack(B)
        path = out / f"{name}.bin"
        raw.tofile(path)
        man[name] = _bin_entry(path, raw, B.shape[0], B.shape[1], how)
    blocks = {}
    for i, b in enumerate(weights["blocks"]):
        mats = {"qkv": (b["qkv"], "[Wq^T | Wk^T | Wv^T]"), "o": (b["o"], "Wo^T"),
                "up": (interleave_up_torch(b["gate"], b["proj"]), "[gate 64 | proj 64] per 128-col tile"),
                "down": (b["down"], "Wdown^T")}
        entry = {}
        for name, (B, how) in mats.items():
            raw = pack(B)
            path = out / f"b{i:02d}_{name}.bin"
            raw.tofile(path)
            entry[name] = _bin_entry(path, raw, B.shape[0], B.shape[1], how)
        for name in NORM_NAMES:
            path = out / f"b{i:02d}_{name}.npy"
            np.save(path, b[name].float().cpu().numpy())
            entry[name] = {"file": path.name, "shape": [int(b[name].numel())], "dtype": "float32"}
        blocks[f"{i:02d}"] = entry
    man["blocks"] = blocks
    man["total_block_bytes"] = sum(e["bytes"] for b in blocks.values() for e in b.values() if "bytes" in e)
    (out / "manifest.json").write_text(json.dumps(man, indent=1))
    return man


def _read_bin(directory, entry, verify):
    path = Path(directory) / entry["file"]
    if not path.exists():
        raise ValueError(f"{path}: missing")
    raw = np.fromfile(path, dtype=np.uint8)
    if raw.size != entry["bytes"] or raw.size != entry["K"] * entry["N"] // 8 * 9:
        raise ValueError(f"{path}: {raw.size} bytes, manifest says {entry['bytes']} for K={entry['K']} N={entry['N']}")
    if verify and _sha256(raw) != entry["sha256"]:
        raise ValueError(f"{path}: sha256 does not match the manifest")
    return raw


def read_manifest(directory, blocks=None, verify=True):
    """The manifest and every file it names, as host arrays: {"manifest", "img_in", "proj_out", "blocks": [{name:
    bytes or array}], "host": {tensor: array}}. `blocks`: indices to read (default: all in the manifest)."""
    d = Path(directory)
    man = json.loads((d / "manifest.json").read_text())
    ids = sorted(int(k) for k in man["blocks"]) if blocks is None else list(blocks)
    out = {"manifest": man, "blocks": []}
    for name in ("img_in", "proj_out"):
        out[name] = _read_bin(d, man[name], verify)
    for i in ids:
        e = man["blocks"][f"{i:02d}"]
        blk = {name: _read_bin(d, e[name], verify) for name in BIN_NAMES}
        for name in NORM_NAMES:
            path = d / e[name]["file"]
            if not path.exists():
                raise ValueError(f"{path}: missing")
            blk[name] = np.load(path).astype(np.float32)
        out["blocks"].append(blk)
    out["host"] = {}
    for name, e in man.get("host", {}).items():
        path = d / e["file"]
        if not path.exists():
            raise ValueError(f"{path}: missing")
        out["host"][name] = np.load(path).astype(np.float32)
    return out


def load_packed(directory, blocks=None, device="cuda", verify=True):
    """Resident native weights for dit.DiT from a packed directory: the bytes go to the device once and are
    converted to the native tile format there (lossless)."""
    host = read_manifest(directory, blocks, verify)
    man = host["manifest"]
    dev = torch.device(device)

    def native(raw, entry, swiglu=False, cols=None):
        t = torch.from_numpy(raw).to(dev)
        K, N = entry["K"], entry["N"]
        if cols is not None and cols < N:    # b_layout is N-tile outer: the first `cols` columns come first
            t, N = t[:K * cols // 8 * 9].contiguous(), cols
        return ops.PackedWeight.from_pack_b(t, K, N, swiglu)

    out = {"blocks": [], "host": host["host"]}
    out["img_in"] = native(host["img_in"], man["img_in"])
    out["proj_out"] = native(host["proj_out"], man["proj_out"], cols=128)
    ids = sorted(int(k) for k in man["blocks"]) if blocks is None else list(blocks)
    for i, blk in zip(ids, host["blocks"]):
        e = man["blocks"][f"{i:02d}"]
        out["blocks"].append({
            "qkv": native(blk["qkv"], e["qkv"]), "o": native(blk["o"], e["o"]),
            "up": native(blk["up"], e["up"], swiglu=True), "down": native(blk["down"], e["down"]),
            "norm_q": torch.from_numpy(blk["norm_q"]).to(dev), "norm_k": torch.from_numpy(blk["norm_k"]).to(dev),
        })
    return out
