"""Activations with outlier channels, through the decode GEMVs (GPTQ and Q4_K) on the GPU.

The decode kernels stage activations as 23-bit integers with one power-of-two exponent per
group of K (the quantisation group for GPTQ, the 256-value super-block for Q4_K), so an
ordinary element keeps about 22 - log2(group max / |x|) bits. LLM activations routinely carry
channels 100-1000x larger than the rest; these tests put such channels into N(0, 1) rows and
check the error on the part of the output that the ordinary channels produce:

    max |y - ref| / max |x_without_outliers @ W|  <  2e-3

with `ref` the oracle's output on the full x (oracle/gptq.py `gptq_matmul`, the restatement of
webtorch/_core.py:4046-4072; oracle/q4k.py `matmul`, webtorch/_core.py:4399-4406 over the
reference dequantiser). Normalising by the outliers' own contribution instead would hide a loss
of precision on everything else.
"""
import numpy as np
import pytest
import torch

from oracle import gptq as og
from oracle import q4k as oq
from webpytorch_b200 import synth
from webpytorch_b200.ggml import ggml_matmul
from webpytorch_b200.qlinear import _gptq_matmul

pytestmark = pytest.mark.gpu
TOL = 2e-3
DEV = "cuda"


def _with_outliers(M, K, seed, dtype=np.float16):
    """N(0, 1) rows with 3 channels at 100x and 3 at 1000x (the same channels in every row, as
    outlier features are); returns (x, x with those channels zeroed)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K)).astype(np.float32)
    ch = rng.choice(K, 6, replace=False)
    x[:, ch[:3]] *= 100.0
    x[:, ch[3:]] *= 1000.0
    x = x.astype(dtype).astype(np.float32)
    xo = x.copy()
    xo[:, ch] = 0.0
    return x, xo


def _bulk_err(y, ref, xo, W):
    base = np.abs(xo.astype(np.float64) @ W.astype(np.float64)).max()
    return float(np.abs(np.asarray(y, np.float64) - ref).max() / base)


@pytest.mark.parametrize("K,N", [(4096, 4096), (14336, 4096)])
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M", [1, 4, 16])
def test_gptq_outlier_channels(K, N, bits, M):
    w = synth.gptq_weights(K, N, bits, 128, seed=K + bits)
    x, xo = _with_outliers(M, K, seed=M + K)
    ref = og.gptq_matmul(x, w["qweight"], w["qzeros"], w["scales"], K, N, 128, bits, 1.0)
    W = og.gptq_dequant(w["qweight"], w["qzeros"], w["scales"], 128, bits, 1.0)
    qw, qz, sc = (torch.from_numpy(w[k]).to(DEV) for k in ("qweight", "qzeros", "scales"))
    y = _gptq_matmul(torch.from_numpy(x).to(DEV).half(), qw, qz, sc, K, N, 128, bits, 1.0).cpu().numpy()
    err = _bulk_err(y, ref, xo, W)
    assert err < TOL, err


@pytest.mark.parametrize("M", [1, 3, 8, 13])
def test_q4k_outlier_channels_fp32_x(M):
    K, N = 4096, 2048
    raw = synth.q4k_weights(N, K, seed=M)
    x, xo = _with_outliers(M, K, seed=M, dtype=np.float32)
    ref = oq.matmul(x, raw.tobytes(), K, N)
    W = oq.dequant(raw.tobytes(), N * K).reshape(N, K)
    rd = torch.from_numpy(raw.reshape(-1)).to(DEV)
    y = ggml_matmul(torch.from_numpy(x).to(DEV), rd, "Q4_K", K, N).cpu().numpy()
    err = _bulk_err(y, ref, xo, W.T)
    assert err < TOL, err


@pytest.mark.parametrize("M", [1, 4, 8, 12])
@pytest.mark.parametrize("bad", [np.inf, -np.inf, np.nan])
def test_gptq_nonfinite_activation_gives_nan_row(M, bad):
    """A token row holding inf or nan gives a NaN output row (the integer staging cannot carry
    non-finite values); every other row is unaffected."""
    K, N = 1024, 256
    w = synth.gptq_weights(K, N, 4, 128, seed=6)
    x = synth.activations(M, K, np.float32, seed=M)
    r = M // 2
    x[r, 300] = bad
    qw, qz, sc = (torch.from_numpy(w[k]).to(DEV) for k in ("qweight", "qzeros", "scales"))
    y = _gptq_matmul(torch.from_numpy(x).to(DEV), qw, qz, sc, K, N, 128, 4, 1.0).cpu().numpy()
    x[r, 300] = 0.0
    ref = og.gptq_matmul(x, w["qweight"], w["qzeros"], w["scales"], K, N, 128, 4, 1.0)
    assert np.isnan(y[r]).all()
    others = [m for m in range(M) if m != r]
    if others:
        d = np.abs(y[others] - ref[others]).max() / np.abs(ref[others]).max()
        assert d < TOL, d


@pytest.mark.parametrize("M", [1, 6])
def test_q4k_nonfinite_activation_gives_nan_row(M):
    K, N = 512, 256
    raw = synth.q4k_weights(N, K, seed=4)
    x = synth.activations(M, K, np.float32, seed=M)
    x[0, 17] = np.nan
    rd = torch.from_numpy(raw.reshape(-1)).to(DEV)
    y = ggml_matmul(torch.from_numpy(x).to(DEV), rd, "Q4_K", K, N).cpu().numpy()
    assert np.isnan(y[0]).all()
    if M > 1:
        ref = oq.matmul(x[1:], raw.tobytes(), K, N)
        assert np.abs(y[1:] - ref).max() / np.abs(ref).max() < TOL
