"""CPU oracle of the reference's NPU attention formats - TEST INFRASTRUCTURE ONLY (tests/ import it; the package never
does).

Restates, on numpy arrays:
  q_pack / kv_pack       the per-head 64-token tile streams its attention kernels read (redline/run_attn.py:29-35 pack_kv,
                         82-85 pack_q_small; run_attn.py:147-150 for several Q tiles): Q tile = to_bfp16(a_layout(Q_t,
                         64, 128)), K tile = to_bfp16(b_layout(K_t^T, 128, 64)), V tile = to_bfp16(b_layout(V_t, 64,
                         128)), per head [K0 V0 K1 V1 ...]
  q_unpack / kv_unpack   their inverses (run_qkv.py:82-88 unpack_head)
  tables / tables_decode the QKV-post kernel's table (run_qkv.py:33-36 _ROWS / _PAIRS, 60-72 qkv_tables) and its inverse
  lim_pack               the per-row key-limit buffer (run_attn.py:87-92 pack_lim)
Pinned against the reference's own outputs in tests/golden (npu_* arrays, made by tests/golden/make_golden.py).
"""

import numpy as np

from . import bfp16_oracle as O

TILE = 64
D = 128
_BLK = np.arange(128)
ROWS = (_BLK // 32)[:, None] * 16 + ((_BLK % 4) // 2)[:, None] * 8 + np.arange(8)[None, :]        # (128, 8)
PAIRS = ((_BLK // 4) % 8)[:, None] * 8 + ((_BLK % 4) % 2)[:, None] * 4 + np.arange(4)[None, :]    # (128, 4)


def q_pack(q):
    """q (H, 64T, 128) -> the Q stream (H * T tiles of 9216 bytes)."""
    return np.concatenate([O.to_bfp16(O.a_layout(np.asarray(q[h], np.float32), TILE, D)) for h in range(len(q))])


def kv_pack(k, v):
    """k, v (H, 64T, 128) -> per head [K0 V0 K1 V1 ...] tile bytes."""
    out = []
    for h in range(len(k)):
        for t in range(0, k.shape[1], TILE):
            out.append(O.to_bfp16(O.b_layout(np.asarray(k[h, t:t + TILE], np.float32).T, D, TILE)))
            out.append(O.to_bfp16(O.b_layout(np.asarray(v[h, t:t + TILE], np.float32), TILE, D)))
    return np.concatenate(out)


def q_unpack(raw, H):
    """The Q stream of H heads -> (H, 64T, 128) float32."""
    per = np.asarray(raw).reshape(H, -1)
    rows = per.shape[1] // 9 * 8 // D
    return np.stack([O.a_unlayout(O.from_bfp16(per[h]), rows, D, TILE, D) for h in range(H)])


def kv_unpack(raw, H):
    """Per-head [K|V] tile streams -> k, v (H, 64T, 128) float32."""
    tiles = np.asarray(raw).reshape(H, -1, 2, TILE * D // 8 * 9)
    k = np.stack([np.concatenate([O.b_unlayout(O.from_bfp16(tiles[h, t, 0]), D, TILE, D, TILE).T
                                  for t in range(tiles.shape[1])]) for h in range(H)])
    v = np.stack([np.concatenate([O.b_unlayout(O.from_bfp16(tiles[h, t, 1]), TILE, D, TILE, D)
                                  for t in range(tiles.shape[1])]) for h in range(H)])
    return k, v


def tables(cos, sin, wq, wk):
    """cos, sin (64T, 64), w_q * log2(e)/sqrt(128) and w_k (128) -> the table (T, 8448) as bf16 bit patterns."""
    T = cos.shape[0] // TILE
    c = np.asarray(cos, np.float32).reshape(T, 64, 64)[:, ROWS[:, :, None], PAIRS[:, None, :]].reshape(T, 128, 32)
    s = np.asarray(sin, np.float32).reshape(T, 64, 64)[:, ROWS[:, :, None], PAIRS[:, None, :]].reshape(T, 128, 32)
    tab = np.empty((T, 128 * 64 + 256), np.float32)
    tab[:, :128 * 64] = np.concatenate([c, s], -1).reshape(T, -1)
    tab[:, 128 * 64:128 * 64 + 128] = wq
    tab[:, 128 * 64 + 128:] = wk
    return O.bf16_bits(O.bf16_round(tab))


def tables_decode(tab_bits):
    """The table (T, 8448) bf16 bits -> cos, sin (64T, 64), w_q, w_k (128) float32."""
    t = O.bf16_from_bits(np.asarray(tab_bits, np.uint16)).astype(np.float32)
    T = t.shape[0]
    cs = t[:, :128 * 64].reshape(T, 128, 2, 8, 4)
    cos = np.empty((T, 64, 64), np.float32)
    sin = np.empty((T, 64, 64), np.float32)
    cos[:, ROWS[:, :, None], PAIRS[:, None, :]] = cs[:, :, 0]
    sin[:, ROWS[:, :, None], PAIRS[:, None, :]] = cs[:, :, 1]
    return cos.reshape(T * 64, 64), sin.reshape(T * 64, 64), t[0, 128 * 64:128 * 64 + 128], t[0, 128 * 64 + 128:]


def lim_pack(lim, mq=64, nt=64):
    """Per-row last visible key (int32) at the start of one tile-sized buffer."""
    buf = np.zeros(mq * nt // 8 * 9, np.uint8)
    buf[:4 * mq] = np.asarray(lim, np.int32).view(np.uint8)
    return buf
