"""The CPU oracle against golden vectors produced by the reference's own code (CPU only)."""
import numpy as np
import pytest

from conftest import golden, golden_files, max_rel_err, same_bits_or_both_nan
from oracle import gptq as og
from oracle import moe as om
from oracle import q4k as oq
from webpytorch_b200 import synth


@pytest.mark.parametrize("name", golden_files("gptq_ref_"))
def test_gptq_dequant_bitexact_vs_reference(name):
    d = golden(name)
    W = og.gptq_dequant(d["qweight"], d["qzeros"], d["scales"], int(d["gs"]), int(d["bits"]), float(d["zoff"]))
    assert W.dtype == np.float32
    assert np.array_equal(W.view(np.uint32), d["W"].view(np.uint32))


@pytest.mark.parametrize("name", golden_files("gptq_ref_"))
def test_gptq_matmul_vs_reference(name):
    d = golden(name)
    K, N, gs, bits = (int(d[k]) for k in ("K", "N", "gs", "bits"))
    for M in (1, 3, 4, 5, 32):
        y = og.quantized_linear(d["x_%d" % M], d["qweight"], d["qzeros"], d["scales"], None, K, N, K, N, gs,
                                bits, 0.0)
        assert max_rel_err(y, d["y_%d" % M]) < 1e-6


@pytest.mark.parametrize("name", golden_files("gptq_autogptq_"))
def test_gptq_autogptq_vs_reference(name):
    d = golden(name)
    K, N, gs, bits = (int(d[k]) for k in ("K", "N", "gs", "bits"))
    y = og.quantized_linear(d["x"].astype(np.float32), d["qweight"], d["qzeros"], d["scales"], d.get("bias"),
                            K, N, K, N, gs, bits, 1.0)
    assert max_rel_err(y, d["y"]) < 1e-6


def test_gptq_quantizer_and_fromlinear_vs_reference():
    d = golden("gptq_fromlinear.npz")
    K, N, Kp, Np, gs, bits = (int(d[k]) for k in ("K", "N", "Kp", "Np", "gs", "bits"))
    W = np.pad(d["weight"], ((0, Kp - K), (0, Np - N)))
    qw, qz, sc, _, _ = og.gptq_quantize(W, gs, bits)
    assert np.array_equal(qw, d["qweight"]) and np.array_equal(qz, d["qzeros"])
    assert np.array_equal(sc.view(np.uint32), d["scales"].astype(np.float32).view(np.uint32))
    y = og.quantized_linear(d["x"], qw, qz, sc, d["bias"], K, N, Kp, Np, gs, bits, 0.0)
    assert max_rel_err(y, d["y"]) < 1e-6


def test_desc_act_restatement_pins_to_reference():
    """With g_idx = arange//gs the desc_act formula is the reference's; with a row permutation
    it equals the plain weight applied to correspondingly permuted activations."""
    d = golden("gptq_autogptq_K512_N192_g128_b4.npz")
    K, N, gs, bits = (int(d[k]) for k in ("K", "N", "gs", "bits"))
    x = d["x"].astype(np.float32)
    y_plain = og.gptq_matmul(x, d["qweight"], d["qzeros"], d["scales"], K, N, gs, bits, 1.0,
                             g_idx=np.arange(K) // gs)
    assert max_rel_err(y_plain + d["bias"], d["y"]) < 1e-6
    rng = np.random.default_rng(5)
    pi = rng.permutation(K)
    qa = og.sort_rows(d["qweight"], pi, bits)           # act-order checkpoint rows
    ga = (np.arange(K) // gs)[pi]
    y_act = og.gptq_matmul(x, qa, d["qzeros"], d["scales"], K, N, gs, bits, 1.0, g_idx=ga)
    x_plain = np.empty_like(x)
    x_plain[:, pi] = x
    y_ref = og.gptq_matmul(x_plain, d["qweight"], d["qzeros"], d["scales"], K, N, gs, bits, 1.0)
    assert max_rel_err(y_act, y_ref) < 1e-5


def test_autogptq_packer_roundtrip():
    rng = np.random.default_rng(3)
    K, N, gs, bits = 256, 64, 128, 4
    q = rng.integers(0, 16, (K, N))
    zp = rng.integers(1, 16, (K // gs, N))
    sc = rng.uniform(0.01, 0.02, (K // gs, N)).astype(np.float32)
    qw, qz, sc16, gidx = og.pack_autogptq(q, sc, zp, gs, bits)
    assert np.array_equal(og.unpack_rows(qw, bits), q)
    assert np.array_equal(og.unpack_cols(qz, bits) + 1, zp)
    assert np.array_equal(gidx, np.arange(K) // gs)


def test_q4k_dequant_bitexact_vs_reference():
    for name in ("q4k_randombytes.npz", "q4k_synth.npz", "q4k_rawbytes_nonfinite.npz"):
        d = golden(name)
        N, K = int(d["N"]), int(d["K"])
        W = oq.dequant(d["raw"].tobytes(), N * K).reshape(N, K)
        assert same_bits_or_both_nan(W, d["W"])


def test_q4k_matmul_vs_reference():
    d = golden("q4k_synth.npz")
    N, K = int(d["N"]), int(d["K"])
    for M in (1, 8, 13):
        y = oq.matmul(d["x_%d" % M], d["raw"].tobytes(), K, N)
        assert max_rel_err(y, d["y_%d" % M]) < 1e-6


def test_q4k_scale_packing_roundtrip():
    rng = np.random.default_rng(0)
    sc = rng.integers(0, 64, (100, 8), dtype=np.uint8)
    m = rng.integers(0, 64, (100, 8), dtype=np.uint8)
    s = synth.pack_q4k_scales(sc, m)
    sc2, m2 = oq.scale_min(s)
    assert np.array_equal(sc2, sc) and np.array_equal(m2, m)


@pytest.mark.parametrize("name", golden_files("moe_"))
def test_moe_vs_reference(name):
    d = golden(name)
    E, top_k, H, I, gs, bits = (int(d[k]) for k in ("E", "top_k", "H", "I", "gs", "bits"))

    def lin(pre, k, Kin, Nout):
        qw, qz, sc = (d["%s_%s_%s" % (pre, k, f)] for f in ("qweight", "qzeros", "scales"))
        return lambda x: og.quantized_linear(x, qw, qz, sc, None, Kin, Nout, Kin, Nout, gs, bits, 1.0)

    experts = [(lin("e%d" % e, "gate", H, I), lin("e%d" % e, "up", H, I), lin("e%d" % e, "down", I, H))
               for e in range(E)]
    shared = shared_gate = None
    if "SI" in d:
        SI = int(d["SI"])
        shared = (lin("shared", "gate", H, SI), lin("shared", "up", H, SI), lin("shared", "down", SI, H))
        shared_gate = (lambda x: x @ d["shared_gate_w"])
    norm = bool(int(d["norm_topk_prob"])) if "norm_topk_prob" in d else True
    y = om.moe_mlp(d["x"], d["logits"], experts, top_k, norm, shared, shared_gate)
    assert max_rel_err(y, d["y"]) < 1e-6


# ---------------------------------------------------------------------------------------
# other GGUF types, the AutoGPTQ writer (fixtures made by the reference)
# ---------------------------------------------------------------------------------------
@pytest.mark.parametrize("name", golden_files("ggml_"))
def test_ggml_oracle_matches_reference_dequant(name):
    from oracle import ggml as ogg
    d = golden(name)
    tname = {8: "Q8_0", 13: "Q5_K", 14: "Q6_K"}[int(d["type_id"])]
    N, K = int(d["N"]), int(d["K"])
    W = ogg.dequant(tname, d["raw"].tobytes(), N * K).reshape(N, K)
    assert same_bits_or_both_nan(W, d["W"])
    for M in (1, 3, 8):
        if "x_%d" % M in d:
            y = ogg.matmul(d["x_%d" % M], d["raw"].tobytes(), tname, K, N)
            assert np.array_equal(y, d["y_%d" % M])


@pytest.mark.parametrize("name", golden_files("gptq_writer_"))
def test_writer_oracle_matches_reference(name):
    d = golden(name)
    gs, bits = int(d["gs"]), int(d["bits"])
    q, sc, zp = og.quantize_raw(d["W"], gs, bits)
    qw, qz, scq, gidx = og.pack_autogptq(q, sc, zp, gs, bits)
    assert np.array_equal(qw, d["qweight"]) and np.array_equal(qz, d["qzeros"])
    assert np.array_equal(scq.view(np.uint16), d["scales"].view(np.uint16))
    assert np.array_equal(gidx, d["g_idx"])
