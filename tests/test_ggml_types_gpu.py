"""GGUF Q8_0 / Q5_K / Q6_K on the GPU: exact dequantisation against the reference's own output
(tests/golden/ggml_*.npz, made by ggufload.dequant), the decode GEMV against the reference's
x @ W.T and, at the config-2 size, against the exact dequant in fp64."""
import numpy as np
import pytest
import torch

from conftest import golden, golden_files, max_rel_err, same_bits_or_both_nan
from webpytorch_b200 import synth
from webpytorch_b200.ggml import GGMLLinear, ggml_dequant, ggml_matmul

pytestmark = pytest.mark.gpu
TOL = 2e-3
DEV = "cuda"
NAMES = {8: "Q8_0", 13: "Q5_K", 14: "Q6_K"}


def _raw(a):
    return torch.from_numpy(np.ascontiguousarray(a).reshape(-1).view(np.uint8)).to(DEV)


@pytest.mark.parametrize("name", golden_files("ggml_"))
def test_dequant_bitexact_vs_reference(name):
    d = golden(name)
    N, K = int(d["N"]), int(d["K"])
    W = ggml_dequant(_raw(d["raw"]), NAMES[int(d["type_id"])], K, N).cpu().numpy()
    assert same_bits_or_both_nan(W, d["W"])


@pytest.mark.parametrize("t", ["Q8_0", "Q5_K", "Q6_K"])
@pytest.mark.parametrize("xdt", [torch.float32, torch.float16, torch.bfloat16])
def test_matmul_vs_reference(t, xdt):
    d = golden("ggml_%s_synth.npz" % t)
    N, K = int(d["N"]), int(d["K"])
    lin = GGMLLinear(d["raw"], t, K, N)
    for M in (1, 3, 8):
        x = torch.from_numpy(d["x_%d" % M]).to(DEV).to(xdt)
        y = lin(x).cpu().numpy()
        ref = d["y_%d" % M] if xdt == torch.float32 else x.float().cpu().numpy() @ d["W"].T
        assert max_rel_err(y, ref) < TOL, (M, max_rel_err(y, ref))


@pytest.mark.parametrize("t", ["Q8_0", "Q5_K", "Q6_K"])
@pytest.mark.parametrize("M", [1, 4, 9])
def test_config2_size_vs_exact_dequant(t, M):
    N, K = 14336, 4096
    raw = synth.ggml_weights(t, N, K, seed=M)
    rd = _raw(raw)
    W = ggml_dequant(rd, t, K, N).double()
    x = torch.randn((M, K), device=DEV, generator=torch.Generator(device=DEV).manual_seed(M))
    bias = torch.randn(N, device=DEV, generator=torch.Generator(device=DEV).manual_seed(M + 1))
    y = ggml_matmul(x, rd, t, K, N, bias=bias)
    ref = x.double() @ W.T + bias.double()
    assert max_rel_err(y.cpu().numpy(), ref.cpu().numpy()) < TOL


def test_unaligned_rows_rejected():
    from webpytorch_b200._ffi import QLError
    raw = synth.ggml_weights("Q6_K", 8, 256, seed=1)      # 210-byte rows: not 4-byte aligned
    lin = GGMLLinear(raw, "Q6_K", 256, 8)
    with pytest.raises(QLError):
        lin(torch.zeros((1, 256), device=DEV))
