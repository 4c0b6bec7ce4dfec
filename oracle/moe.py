"""MoE expert-block oracle (numpy) — test infrastructure, restating webtorch/lm_engine.py.

`moe_mlp` follows lm_engine.py:294-329 with the router replaced by given logits (the
reference's own test stub does the same): float64 softmax over experts (_softmax_rows,
lm_engine.py:331-333), top-k by argpartition, optional renormalisation, then for every expert
with routed tokens `down(silu(gate(x)) * up(x))` weighted and scatter-added.
"""
import numpy as np


def softmax_rows(x):
    """lm_engine.py:331-333."""
    x = np.asarray(x, np.float64)
    e = np.exp(x - x.max(1, keepdims=True))
    return e / e.sum(1, keepdims=True)


def route(logits, top_k, norm_topk_prob=True):
    """Top-k experts and their weights per token (lm_engine.py:301-307)."""
    probs = softmax_rows(logits)
    topk_idx = np.argpartition(-probs, top_k - 1, axis=1)[:, :top_k]
    topk_w = np.take_along_axis(probs, topk_idx, axis=1)
    if norm_topk_prob:
        topk_w = topk_w / topk_w.sum(1, keepdims=True)
    return topk_idx, topk_w


def silu(x):
    """x * sigmoid(x) (webtorch/_core.py:502-503), in float32."""
    x = np.asarray(x, np.float32)
    with np.errstate(over="ignore"):         # exp(-x) -> inf gives silu -> -0, as in the reference
        return (x * (1.0 / (1.0 + np.exp(-x)))).astype(np.float32)


def moe_mlp(x, logits, experts, top_k, norm_topk_prob=True, shared=None, shared_gate=None):
    """x [T, H] float32; experts[e] = (gate, up, down) callables mapping float32 arrays;
    shared = (gate, up, down) or None; shared_gate = callable x -> [T, 1] logits or None.
    Returns float32 [T, H] (lm_engine.py:309-328)."""
    x = np.asarray(x, np.float32)
    T, H = x.shape
    topk_idx, topk_w = route(logits, top_k, norm_topk_prob)
    out = np.zeros((T, H), np.float32)
    for e in range(len(experts)):
        rows, slot = np.where(topk_idx == e)
        if len(rows) == 0:
            continue
        xe = x[rows]
        gate, up, down = experts[e]
        ye = down(silu(gate(xe)) * up(xe))
        w = topk_w[rows, slot].astype(np.float32)
        ye = ye * w.reshape(-1, 1)
        out[rows] = out[rows] + ye
    if shared is not None:
        # lm_engine.py:322-328: shared expert over every token, optionally sigmoid-gated
        sg, su, sd = shared
        ys = sd(silu(sg(x)) * su(x)).astype(np.float32)
        if shared_gate is not None:
            g = 1.0 / (1.0 + np.exp(-np.asarray(shared_gate(x))))
            ys = ys * g
        out = out + ys
    return out.astype(np.float32)
