"""Decode-layer oracle (numpy) — test infrastructure, restating the reference's layer math for one
token with a growing KV cache: webtorch/lm_engine.py:62-64 (`_rms`), 66-70 (`_rope`), 72-74
(`_rot`), 84-87 (`_mlp`), 89-107 (`_block` at T = 1), in float32 as the reference's tensors are.
The linears are callables (the GPTQ oracle's quantized_linear on the layer's packed weights).
"""
import numpy as np

from .moe import silu


def rms(x, w, eps):
    """(x / sqrt(mean(x * x) + eps)) * w over the last axis (lm_engine.py:62-64)."""
    x = np.asarray(x, np.float32)
    return ((x / np.sqrt((x * x).mean(axis=-1, keepdims=True) + np.float32(eps))) * w).astype(np.float32)


def rope(x, pos, theta):
    """x [heads, HD] rotated at position pos: x * cos + rot(x) * sin, rot(x) = [-x2, x1]
    (lm_engine.py:66-74; angles in float64, tables rounded to float32)."""
    HD = x.shape[-1]
    inv = 1.0 / (theta ** (np.arange(0, HD, 2, dtype=np.float64) / HD))
    ang = np.float64(pos) * inv
    emb = np.concatenate([ang, ang])
    cos, sin = np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)
    rot = np.concatenate([-x[:, HD // 2:], x[:, :HD // 2]], axis=-1)
    return (x * cos + rot * sin).astype(np.float32)


def layer_step(h, lay, cache, pos, NH, NKV, HD, theta, eps):
    """One token through one layer. lay: dict of callables q, k, v, o, gate, up, down (float32
    [1, in] -> [1, out]) and arrays in_ln, post_ln; cache: dict with lists K, V of [NKV, HD]
    rows (appended). Returns the new h [1, H]."""
    x = rms(h, lay["in_ln"], eps)
    q = lay["q"](x).reshape(NH, HD)
    k = lay["k"](x).reshape(NKV, HD)
    v = lay["v"](x).reshape(NKV, HD)
    q, k = rope(q, pos, theta), rope(k, pos, theta)
    cache["K"].append(k)
    cache["V"].append(v)
    K = np.stack(cache["K"])          # [T, NKV, HD]
    V = np.stack(cache["V"])
    g = NH // NKV
    o = np.empty((NH, HD), np.float32)
    for hh in range(NH):
        s = (K[:, hh // g] @ q[hh]) * np.float32(1.0 / np.sqrt(HD))
        p = np.exp(s - s.max())
        p = p / p.sum()
        o[hh] = p @ V[:, hh // g]
    h = (h + lay["o"](o.reshape(1, NH * HD))).astype(np.float32)
    x = rms(h, lay["post_ln"], eps)
    return (h + lay["down"](silu(lay["gate"](x)) * lay["up"](x))).astype(np.float32)
