"""GPTQ qlinear on the GPU against the reference's outputs (golden fixtures) and the oracle.

Tolerances: dequantised weights bit-exact; fp32 outputs within max relative error 2e-3
(max|got-ref| / max|ref|, the reference's own metric); fp16 / bf16 outputs add their own
rounding (2^-11 / 2^-8 relative).
"""
import numpy as np
import pytest
import torch

from conftest import golden, golden_files, max_rel_err
from oracle import gptq as og
from webpytorch_b200 import synth
from webpytorch_b200.qlinear import QuantizedLinear, _gptq_matmul, gptq_dequant

pytestmark = pytest.mark.gpu
TOL = 2e-3
OUT_TOL = {torch.float32: TOL, torch.float16: TOL + 2 ** -11, torch.bfloat16: TOL + 2 ** -8}
DEV = "cuda"


def _t(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    return t if dtype is None else t.to(dtype)


@pytest.mark.parametrize("name", golden_files("gptq_ref_"))
def test_dequant_bitexact_reference_quantizer(name):
    d = golden(name)
    K, N, gs, bits = (int(d[k]) for k in ("K", "N", "gs", "bits"))
    W = gptq_dequant(_t(d["qweight"]), _t(d["qzeros"]), _t(d["scales"]), K, N, gs, bits, 0.0)
    assert np.array_equal(W.cpu().numpy().view(np.uint32), d["W"].view(np.uint32))


@pytest.mark.parametrize("name", golden_files("gptq_autogptq_"))
def test_dequant_bitexact_autogptq(name):
    d = golden(name)
    K, N, gs, bits = (int(d[k]) for k in ("K", "N", "gs", "bits"))
    W = gptq_dequant(_t(d["qweight"]), _t(d["qzeros"]), _t(d["scales"]), K, N, gs, bits, 1.0)
    ref = og.gptq_dequant(d["qweight"], d["qzeros"], d["scales"], gs, bits, 1.0)
    assert np.array_equal(W.cpu().numpy().view(np.uint32), ref.view(np.uint32))


def test_dequant_bitexact_desc_act():
    w = synth.gptq_weights(512, 256, 4, 128, seed=4, desc_act=True)
    W = gptq_dequant(_t(w["qweight"]), _t(w["qzeros"]), _t(w["scales"]), 512, 256, 128, 4, 1.0,
                     g_idx=_t(w["g_idx"]))
    ref = og.gptq_dequant(w["qweight"], w["qzeros"], w["scales"], 128, 4, 1.0, g_idx=w["g_idx"])
    assert np.array_equal(W.cpu().numpy().view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("name", golden_files("gptq_ref_"))
@pytest.mark.parametrize("xdt", [torch.float32, torch.float16, torch.bfloat16])
def test_matmul_vs_reference_quantizer_outputs(name, xdt):
    d = golden(name)
    K, N, gs, bits = (int(d[k]) for k in ("K", "N", "gs", "bits"))
    ql = QuantizedLinear(d["qweight"], d["qzeros"], d["scales"], np.zeros(N, np.float32), K, N, K, N, gs, bits)
    for M in (1, 3, 4, 5, 32):
        x = d["x_%d" % M]
        y = ql(_t(x, xdt)).cpu().numpy()
        # the kernel sees x rounded to xdt; the reference saw fp32 x
        ref = d["y_%d" % M] if xdt == torch.float32 else og.quantized_linear(
            _t(x, xdt).float().cpu().numpy(), d["qweight"], d["qzeros"], d["scales"], None, K, N, K, N, gs, bits, 0.0)
        assert max_rel_err(y, ref) < TOL, (M, max_rel_err(y, ref))


@pytest.mark.parametrize("name", golden_files("gptq_autogptq_"))
@pytest.mark.parametrize("odt", [torch.float32, torch.float16, torch.bfloat16])
def test_matmul_vs_reference_autogptq(name, odt):
    d = golden(name)
    gs, bits = int(d["gs"]), int(d["bits"])
    ql = QuantizedLinear.from_autogptq(d["qweight"], d["qzeros"], d["scales"], d.get("bias"), gs, bits)
    y = ql(_t(d["x"]), out_dtype=odt).float().cpu().numpy()
    assert max_rel_err(y, d["y"]) < OUT_TOL[odt]


def test_from_linear_padding_and_bias_vs_reference():
    d = golden("gptq_fromlinear.npz")

    class Lin:
        pass
    lin = Lin()
    lin.weight = d["weight"]
    lin.bias = d["bias"]
    ql = QuantizedLinear.from_linear(lin, group_size=int(d["gs"]), bits=int(d["bits"]))
    assert (ql.Kp, ql.Np) == (int(d["Kp"]), int(d["Np"]))
    assert np.array_equal(ql.qweight.cpu().numpy(), d["qweight"])
    assert np.array_equal(ql.qzeros.cpu().numpy(), d["qzeros"])
    assert np.array_equal(ql.scales.cpu().numpy().view(np.uint32), d["scales"].view(np.uint32))
    y = ql(torch.from_numpy(d["x"]))           # host tensor in -> host tensor out
    assert y.device.type == "cpu" and tuple(y.shape) == tuple(d["y"].shape)
    assert max_rel_err(y.numpy(), d["y"]) < TOL


@pytest.mark.parametrize("bits,gs", [(4, 128), (8, 128), (4, 32), (8, 64)])
@pytest.mark.parametrize("M", [1, 7, 16, 17, 40])
@pytest.mark.parametrize("N", [384, 200])    # 384: TMA-fed GEMV; 200 (not a multiple of 32): register-fed
def test_desc_act_vs_oracle(bits, gs, M, N):
    K = 1024
    w = synth.gptq_weights(K, N, bits, gs, seed=M + bits, desc_act=True)
    x = synth.activations(M, K, np.float16, seed=M)
    ql = QuantizedLinear.from_autogptq(w["qweight"], w["qzeros"], w["scales"], None, gs, bits, g_idx=w["g_idx"])
    assert ql.x_perm is not None
    y = ql(_t(x)).cpu().numpy()
    ref = og.gptq_matmul(x.astype(np.float32), w["qweight"], w["qzeros"], w["scales"], K, N, gs, bits, 1.0,
                         g_idx=w["g_idx"])
    assert max_rel_err(y, ref) < TOL


def test_unequal_groups_rejected():
    K, N = 256, 64
    w = synth.gptq_weights(K, N, 4, 128, seed=1)
    g = np.zeros(K, np.int32)
    g[:200] = 1
    with pytest.raises(NotImplementedError):
        QuantizedLinear.from_autogptq(w["qweight"], w["qzeros"], w["scales"], None, 128, 4, g_idx=g)


# config-1 shapes at full size; checked against the exact dequant (bit-exact above) in fp64
@pytest.mark.parametrize("K,N", [(4096, 4096), (4096, 11008), (11008, 4096), (4096, 14336), (14336, 4096)])
@pytest.mark.parametrize("bits", [4, 8])
def test_config1_full_size(K, N, bits):
    w = synth.gptq_weights(K, N, bits, 128, seed=K + N + bits)
    qw, qz, sc = _t(w["qweight"]), _t(w["qzeros"]), _t(w["scales"])
    W = gptq_dequant(qw, qz, sc, K, N, 128, bits, 1.0).double()
    for M in (1, 4, 16):
        x = _t(synth.activations(M, K, np.float16, seed=M))
        y = _gptq_matmul(x, qw, qz, sc, K, N, 128, bits, 1.0)
        ref = x.double() @ W
        assert max_rel_err(y.cpu().numpy(), ref.cpu().numpy()) < TOL
    # full-size spot check of the exact dequant against the oracle on a column slab
    ref_w = og.gptq_dequant(w["qweight"][:, :256], w["qzeros"][:, :256 // (32 // bits)], w["scales"][:, :256],
                            128, bits, 1.0)
    assert np.array_equal(W[:, :256].float().cpu().numpy().view(np.uint32), ref_w.view(np.uint32))


def test_deterministic_and_stream_ordered():
    K, N = 4096, 4096
    w = synth.gptq_weights(K, N, 4, 128, seed=9)
    ql = QuantizedLinear.from_autogptq(w["qweight"], w["qzeros"], w["scales"], None, 128, 4)
    x = _t(synth.activations(3, K, np.float16, seed=2))
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        y1 = ql(x)
        y2 = ql(x)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)


@pytest.mark.parametrize("M", [4, 8, 12])
def test_row_scales_far_outside_fp16_range(M):
    """Whole rows scaled by 1e6 and by 1e-6 are staged exactly (every group takes its own power
    of two), per-row error within 2e-3 of the row's own output. Up to 4 tokens the CTAs stage
    the activations themselves, above that they are staged once in global memory."""
    K, N = 1024, 256
    w = synth.gptq_weights(K, N, 4, 128, seed=5)
    x = synth.activations(M, K, np.float32, seed=3)
    x[0] *= 1e6
    x[1] *= 1e-6
    x[2] *= 3e4
    ql = QuantizedLinear.from_autogptq(w["qweight"], w["qzeros"], w["scales"], None, 128, 4)
    y = ql(_t(x)).cpu().numpy()
    ref = og.gptq_matmul(x, w["qweight"], w["qzeros"], w["scales"], K, N, 128, 4, 1.0)
    for m in range(M):
        assert max_rel_err(y[m], ref[m]) < TOL, m


def test_isolated_extreme_element_limits_only_its_group():
    """One element 3e5 times the rest dominates its own 128-value group (the group's other values
    keep about 4 bits), but every other group of the row keeps full precision: the error on the
    output without that group's contribution stays within 2e-3 of the row's ordinary output."""
    K, N = 1024, 256
    w = synth.gptq_weights(K, N, 4, 128, seed=5)
    x = synth.activations(2, K, np.float32, seed=3)
    x[1, 5] = 3e5
    ql = QuantizedLinear.from_autogptq(w["qweight"], w["qzeros"], w["scales"], None, 128, 4)
    y = ql(_t(x)).cpu().numpy()
    ref = og.gptq_matmul(x, w["qweight"], w["qzeros"], w["scales"], K, N, 128, 4, 1.0)
    W = og.gptq_dequant(w["qweight"], w["qzeros"], w["scales"], 128, 4, 1.0).astype(np.float64)
    base = np.abs(x[1, 128:].astype(np.float64) @ W[128:]).max()
    # the outlier's group: each value within half a step (2^-22 of the group maximum) of x, plus
    # the fp32 rounding of the reference's own sum over a 3e5-sized term
    bound = 2.0 ** -22 * 3e5 * np.abs(W[:128]).sum(0).max() + 1e-6 * np.abs(ref[1]).max()
    assert np.abs(y[1] - ref[1]).max() <= bound + TOL * base
    assert max_rel_err(y[0], ref[0]) < TOL


@pytest.mark.parametrize("M", [8, 12])
def test_staged_activations_extreme_and_nonfinite_rows(M):
    """Decode calls of more than 4 tokens stage the activations once in global memory: rows far
    outside fp16 range are scaled exactly, a row holding inf / nan gives a NaN output row."""
    K, N = 1024, 256
    w = synth.gptq_weights(K, N, 4, 128, seed=6)
    x = synth.activations(M, K, np.float32, seed=M)
    x[0] *= 1e6
    x[1] *= 1e-6
    x[3, 7] = np.inf
    ql = QuantizedLinear.from_autogptq(w["qweight"], w["qzeros"], w["scales"], None, 128, 4)
    y = ql(_t(x)).cpu().numpy()
    ref = og.gptq_matmul(np.nan_to_num(x, posinf=0.0), w["qweight"], w["qzeros"], w["scales"], K, N, 128, 4, 1.0)
    assert np.isnan(y[3]).all()
    for m in [r for r in range(M) if r != 3]:
        assert max_rel_err(y[m], ref[m]) < TOL, m


def test_empty_batch():
    w = synth.gptq_weights(256, 64, 4, 128, seed=1)
    ql = QuantizedLinear.from_autogptq(w["qweight"], w["qzeros"], w["scales"], None, 128, 4)
    y = ql(torch.zeros((0, 256), device=DEV))
    assert tuple(y.shape) == (0, 64)


# ---------------------------------------------------------------------------------------
# tensor-core prefill path (M >= 17)
# ---------------------------------------------------------------------------------------
@pytest.mark.parametrize("bits,gs", [(4, 128), (8, 128), (4, 32), (4, 64), (8, 32)])
@pytest.mark.parametrize("M", [17, 40, 64, 128, 129, 300])
def test_gemm_path_vs_oracle(bits, gs, M):
    K, N = 512, 384
    w = synth.gptq_weights(K, N, bits, gs, seed=M + bits + gs)
    x = synth.activations(M, K, np.float32, seed=M)
    ql = QuantizedLinear.from_autogptq(w["qweight"], w["qzeros"], w["scales"], None, gs, bits)
    y = ql(_t(x)).cpu().numpy()
    ref = og.gptq_matmul(x, w["qweight"], w["qzeros"], w["scales"], K, N, gs, bits, 1.0)
    assert max_rel_err(y, ref) < TOL
    from webpytorch_b200 import _ffi
    assert _ffi.load().ql_device_status() == 0


@pytest.mark.parametrize("M", [64, 200])
def test_gemm_path_desc_act_bias_ragged_n(M):
    K, N = 768, 200                    # N not a multiple of the 128-column tile
    w = synth.gptq_weights(K, N, 4, 128, seed=M, desc_act=True)
    x = synth.activations(M, K, np.float16, seed=M + 1)
    bias = np.random.default_rng(M).standard_normal(N).astype(np.float32)
    ql = QuantizedLinear.from_autogptq(w["qweight"], w["qzeros"], w["scales"], bias, 128, 4, g_idx=w["g_idx"])
    for odt in (torch.float32, torch.bfloat16):
        y = ql(_t(x), out_dtype=odt).float().cpu().numpy()
        ref = og.gptq_matmul(x.astype(np.float32), w["qweight"], w["qzeros"], w["scales"], K, N, 128, 4, 1.0,
                             g_idx=w["g_idx"]) + bias
        assert max_rel_err(y, ref) < OUT_TOL[odt]


@pytest.mark.parametrize("K,N", [(4096, 11008), (3584, 18944)])
@pytest.mark.parametrize("M", [64, 128, 512, 2048])
def test_config3_full_size(K, N, M):
    """Config 3 (desc_act, bf16 x) at full size against the exact dequant in fp64."""
    w = synth.gptq_weights(K, N, 4, 128, seed=K + M, desc_act=True)
    ql = QuantizedLinear.from_autogptq(w["qweight"], w["qzeros"], w["scales"], None, 128, 4, g_idx=w["g_idx"])
    x = torch.randn((M, K), device=DEV, generator=torch.Generator(device=DEV).manual_seed(M)).to(torch.bfloat16)
    y = ql(x)
    W = gptq_dequant(_t(w["qweight"]), _t(w["qzeros"]), _t(w["scales"]), K, N, 128, 4, 1.0,
                     g_idx=_t(w["g_idx"])).double()
    ref = x.double() @ W
    assert max_rel_err(y.cpu().numpy(), ref.cpu().numpy()) < TOL
