"""The decode step (fused RMSNorm -> QKV GEMV, decode attention, O GEMV + residual, fused RMSNorm
-> gate|up GEMV, SwiGLU -> down GEMV + residual), eager and graph-replayed, against the numpy
restatement of the reference's layer (oracle/decode.py, webtorch/lm_engine.py:62-107) over
several tokens; and the fused linear's options one by one against the oracle."""
import numpy as np
import pytest
import torch

from conftest import max_rel_err
from oracle import decode as odec
from oracle import gptq as og
from oracle import moe as om
from webpytorch_b200 import synth
from webpytorch_b200.decode import DecodeLayer, DecodeStack, fused_linear
from webpytorch_b200.qlinear import QuantizedLinear

pytestmark = pytest.mark.gpu
TOL = 2e-3
DEV = "cuda"


def _lin(rng, K, N, bits=4, bias=False):
    w = synth.gptq_weights(K, N, bits, 128, rng=rng)
    b = (rng.standard_normal(N) * 0.1).astype(np.float32) if bias else None
    ql = QuantizedLinear.from_autogptq(w["qweight"], w["qzeros"], w["scales"], b, 128, bits, device=DEV)
    ref = lambda x, w=w, b=b, K=K, N=N: og.quantized_linear(x, w["qweight"], w["qzeros"], w["scales"], b, K, N, K, N,
                                                           128, bits, 1.0)
    return ql, ref


@pytest.mark.parametrize("M", [1, 3, 7])
def test_fused_linear_options_vs_oracle(M):
    rng = np.random.default_rng(M)
    K, N = 1024, 512
    ql, ref = _lin(rng, K, N, bias=True)
    x = rng.standard_normal((M, K)).astype(np.float32) * 3
    w = rng.uniform(0.5, 1.5, K).astype(np.float32)
    res = rng.standard_normal((M, N)).astype(np.float32)
    xd, wd, rd = (torch.from_numpy(a).to(DEV) for a in (x, w, res))
    y = fused_linear(xd, ql, norm_weight=wd, norm_eps=1e-6, residual=rd).cpu().numpy()
    assert max_rel_err(y, ref(odec.rms(x, w, 1e-6)) + res) < TOL
    # SwiGLU prologue: x rows hold [gate | up] (K each)
    gu = rng.standard_normal((M, 2 * K)).astype(np.float32)
    y2 = fused_linear(torch.from_numpy(gu).to(DEV), ql, glu=K).cpu().numpy()
    assert max_rel_err(y2, ref(om.silu(gu[:, :K]) * gu[:, K:])) < TOL
    # residual aliasing the output
    out = rd.clone()
    fused_linear(xd, ql, residual=out, out=out)
    assert max_rel_err(out.cpu().numpy(), ref(x) + res) < TOL


def _model(L=2, H=256, NH=4, NKV=2, HD=64, I=512, seed=0):
    rng = np.random.default_rng(seed)
    layers, refs = [], []
    for _ in range(L):
        q, rq = _lin(rng, H, NH * HD, bias=True)
        k, rk = _lin(rng, H, NKV * HD, bias=True)
        v, rv = _lin(rng, H, NKV * HD, bias=True)
        o, ro = _lin(rng, NH * HD, H)
        g, rg = _lin(rng, H, I)
        u, ru = _lin(rng, H, I)
        d, rd = _lin(rng, I, H)
        in_ln = rng.uniform(0.5, 1.5, H).astype(np.float32)
        post_ln = rng.uniform(0.5, 1.5, H).astype(np.float32)
        layers.append(DecodeLayer(q, k, v, o, g, u, d, in_ln, post_ln))
        refs.append({"q": rq, "k": rk, "v": rv, "o": ro, "gate": rg, "up": ru, "down": rd, "in_ln": in_ln,
                     "post_ln": post_ln})
    return layers, refs, (H, NH, NKV, HD)


@pytest.mark.parametrize("graph", [False, True])
def test_decode_stack_vs_oracle(graph):
    layers, refs, (H, NH, NKV, HD) = _model()
    theta, eps, lmax = 1e6, 1e-6, 16
    stack = DecodeStack(layers, H, NH, NKV, HD, lmax, theta, eps, graph=graph)
    caches = [{"K": [], "V": []} for _ in refs]
    rng = np.random.default_rng(9)
    for pos in range(4):
        e = rng.standard_normal(H).astype(np.float32)
        y = stack.step(e, pos).cpu().numpy()
        h = e.reshape(1, H)
        for lay, c in zip(refs, caches):
            h = odec.layer_step(h, lay, c, pos, NH, NKV, HD, theta, eps)
        assert max_rel_err(y, h) < TOL, (pos, max_rel_err(y, h))


def test_graph_replay_equals_eager():
    layers, _, (H, NH, NKV, HD) = _model(seed=3)
    a = DecodeStack(layers, H, NH, NKV, HD, 8, graph=False)
    b = DecodeStack(layers, H, NH, NKV, HD, 8, graph=True)
    rng = np.random.default_rng(4)
    for pos in range(3):
        e = rng.standard_normal(H).astype(np.float32)
        ya = a.step(e, pos).clone()
        yb = b.step(e, pos).clone()
        assert torch.equal(ya, yb), pos


@pytest.mark.parametrize("graph", [False, True])
def test_programmatic_launch_equals_plain(graph):
    """The step chained by programmatic dependent launch (the default) gives bit-identical
    results to plain launches: every kernel waits for the previous one's outputs."""
    layers, _, (H, NH, NKV, HD) = _model(seed=5)
    a = DecodeStack(layers, H, NH, NKV, HD, 8, graph=graph, pdl=False)
    b = DecodeStack(layers, H, NH, NKV, HD, 8, graph=graph, pdl=True)
    rng = np.random.default_rng(6)
    for pos in range(3):
        e = rng.standard_normal(H).astype(np.float32)
        ya = a.step(e, pos).clone()
        yb = b.step(e, pos).clone()
        assert torch.equal(ya, yb), pos


def test_position_outside_cache_rejected():
    layers, _, (H, NH, NKV, HD) = _model(L=1)
    s = DecodeStack(layers, H, NH, NKV, HD, 4, graph=False)
    with pytest.raises(ValueError):
        s.step(np.zeros(H, np.float32), 4)
