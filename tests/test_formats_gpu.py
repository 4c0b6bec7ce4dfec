"""Quantize-on-load, the AutoGPTQ writer and the checkpoint loaders on the GPU.

* ql_gptq_quantize against the reference writer's own output (tests/golden/gptq_writer_*.npz,
  made by webtorch/quantize.py `_quantize_raw` + `_pack_autogptq`): bit-identical.
* write_autogptq -> safetensors -> load_autogptq_linear, including an act-order (desc_act)
  checkpoint whose g_idx the reference would ignore, against the oracle.
* GGUF: a dense Q4_K weight and a stacked Q6_K expert tensor from a fixture file, through
  gguf_linear / gguf_experts, against the oracle's x @ W.T.
"""
import json

import numpy as np
import pytest
import torch

from conftest import golden, golden_files, max_rel_err
from oracle import ggml as ogg
from oracle import gptq as og
from webpytorch_b200 import formats

pytestmark = pytest.mark.gpu
TOL = 2e-3
DEV = "cuda"


@pytest.mark.parametrize("name", golden_files("gptq_writer_"))
def test_quantize_kernel_matches_reference_writer(name):
    d = golden(name)
    gs, bits = int(d["gs"]), int(d["bits"])
    for wdt in (torch.float16, torch.float32):
        p = formats.quantize_autogptq(torch.from_numpy(d["W"]).to(wdt), gs, bits)
        assert np.array_equal(p["qweight"].cpu().numpy(), d["qweight"])
        assert np.array_equal(p["qzeros"].cpu().numpy(), d["qzeros"])
        assert np.array_equal(p["scales"].cpu().numpy().view(np.uint16), d["scales"].view(np.uint16))
        assert np.array_equal(p["g_idx"].cpu().numpy(), d["g_idx"])


@pytest.mark.parametrize("gs,bits", [(32, 4), (128, 4), (64, 8)])
def test_quantize_kernel_reference_packing_matches_oracle(gs, bits):
    """zero_store_offset 0 and fp32 scales: the reference's own `_gptq_quantize` packing (float32
    weights), as QuantizedLinear.from_linear uses it."""
    rng = np.random.default_rng(gs + bits)
    K, N = 512, 96
    W = (rng.standard_normal((K, N)) * 0.1).astype(np.float32)
    qw, qz, sc, _, _ = og.gptq_quantize(W, gs, bits)
    p = formats.quantize_autogptq(torch.from_numpy(np.ascontiguousarray(W.T)), gs, bits, zero_store_offset=0,
                                  scales_dtype=torch.float32)
    assert np.array_equal(p["qweight"].cpu().numpy(), qw)
    assert np.array_equal(p["qzeros"].cpu().numpy(), qz)
    assert np.array_equal(p["scales"].cpu().numpy().view(np.uint32), sc.view(np.uint32))


def test_write_then_load_autogptq_checkpoint(tmp_path):
    rng = np.random.default_rng(3)
    K, N, gs, bits = 1024, 384, 128, 4
    W = (rng.standard_normal((N, K)) * 0.05).astype(np.float16)
    bias = rng.standard_normal(N).astype(np.float32)
    cfg = formats.write_autogptq(str(tmp_path / "model.safetensors"), {"model.layers.0.mlp.up_proj": W}, gs, bits,
                                 biases={"model.layers.0.mlp.up_proj": bias})
    (tmp_path / "config.json").write_text(json.dumps({"quantization_config": cfg}))
    st = formats.SafeTensorsDir(str(tmp_path))
    g, b_, da = formats.autogptq_config(st.config())
    assert (g, b_, da) == (gs, bits, False)
    ql = formats.load_autogptq_linear(st, "model.layers.0.mlp.up_proj", g, b_)
    x = rng.standard_normal((3, K)).astype(np.float32)
    y = ql(torch.from_numpy(x).to(DEV)).cpu().numpy()
    ref = og.gptq_matmul(x, st.numpy("model.layers.0.mlp.up_proj.qweight"), st.numpy("model.layers.0.mlp.up_proj.qzeros"),
                         st.numpy("model.layers.0.mlp.up_proj.scales"), K, N, gs, bits, 1.0) \
        + st.numpy("model.layers.0.mlp.up_proj.bias").astype(np.float32)
    assert max_rel_err(y, ref) < TOL
    # and the quantised weight tracks the dense one (4-bit, group 128: about 10 % of the output's
    # scale in the worst element, correlation close to 1)
    yq = y - st.numpy("model.layers.0.mlp.up_proj.bias").astype(np.float32)
    yd = x @ W.astype(np.float32).T
    assert max_rel_err(yq, yd) < 0.25 and np.corrcoef(yq.ravel(), yd.ravel())[0, 1] > 0.99


def test_load_act_order_checkpoint(tmp_path):
    """An AutoGPTQ desc_act checkpoint (g_idx a permutation of k // gs, rows stored in that
    order): the loader passes g_idx on and the result matches the oracle's g_idx-aware unpack."""
    from webpytorch_b200 import synth
    K, N, gs, bits = 1024, 256, 128, 4
    w = synth.gptq_weights(K, N, bits, gs, seed=11, desc_act=True)
    formats.write_safetensors(str(tmp_path / "model.safetensors"),
                              {"l.qweight": w["qweight"], "l.qzeros": w["qzeros"], "l.scales": w["scales"],
                               "l.g_idx": w["g_idx"]})
    st = formats.SafeTensorsDir(str(tmp_path))
    ql = formats.load_autogptq_linear(st, "l", gs, bits)
    assert ql.x_perm is not None
    x = np.random.default_rng(1).standard_normal((5, K)).astype(np.float32)
    y = ql(torch.from_numpy(x).to(DEV)).cpu().numpy()
    ref = og.gptq_matmul(x, w["qweight"], w["qzeros"], w["scales"], K, N, gs, bits, 1.0, g_idx=w["g_idx"])
    assert max_rel_err(y, ref) < TOL


def test_gguf_dense_and_stacked_experts(tmp_path):
    d = golden("gguf_parse.npz")
    p = tmp_path / "m.gguf"
    p.write_bytes(d["gguf"].tobytes())
    gg = formats.GGUFFile(str(p))
    x = np.random.default_rng(2).standard_normal((3, 512)).astype(np.float32)
    lin = formats.gguf_linear(gg, "blk.0.attn_q.weight")
    y = lin(torch.from_numpy(x).to(DEV)).cpu().numpy()
    assert max_rel_err(y, x @ d["W_q4"].T) < TOL
    exps = formats.gguf_experts(gg, "blk.0.ffn_gate_exps.weight")
    assert len(exps) == 4
    for e, lin_e in enumerate(exps):
        ye = lin_e(torch.from_numpy(x).to(DEV)).cpu().numpy()
        assert max_rel_err(ye, x @ d["W_q6"][e].T) < TOL, e
    gg.close()
