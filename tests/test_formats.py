"""On-disk formats on the host (no GPU): the GGUF parser against the reference's own parse of a
fixture file (tests/golden/gguf_parse.npz, made by ggufload.parse_header), safetensors write /
read round trips including a sharded checkpoint, and the AutoGPTQ config."""
import json
import os

import numpy as np
import pytest
import torch

from conftest import golden, same_bits_or_both_nan
from oracle import ggml as ogg
from webpytorch_b200 import formats


@pytest.fixture()
def gguf_file(tmp_path):
    d = golden("gguf_parse.npz")
    p = tmp_path / "m.gguf"
    p.write_bytes(d["gguf"].tobytes())
    return str(p), d


def test_gguf_header_matches_reference_parse(gguf_file):
    path, d = gguf_file
    gg = formats.GGUFFile(path)
    assert gg.version == int(d["version"])
    assert gg.data_start == int(d["data_start"])
    ref_meta = json.loads(str(d["meta"]))
    assert set(gg.metadata) == set(ref_meta)
    for k, v in ref_meta.items():
        got = gg.metadata[k]
        if isinstance(v, float):
            assert got == pytest.approx(v, rel=0, abs=0)
        else:
            assert got == v, k
    names = json.loads(str(d["names"]))
    dims = json.loads(str(d["dims"]))
    assert list(gg.tensors) == names
    for i, n in enumerate(names):
        t = gg.tensors[n]
        assert t["dims"] == dims[i] and t["type"] == int(d["types"][i]) and t["offset"] == int(d["offsets"][i])
    gg.close()


def test_gguf_tensor_bytes_and_slicing(gguf_file):
    path, d = gguf_file
    gg = formats.GGUFFile(path)
    assert np.array_equal(np.frombuffer(gg.raw("blk.0.attn_norm.weight"), np.float32), d["norm"])
    assert gg.shape("blk.0.attn_q.weight") == (48, 512) and gg.type_name("blk.0.attn_q.weight") == "Q4_K"
    W = ogg.dequant("Q4_K", bytes(gg.raw("blk.0.attn_q.weight")), 48 * 512).reshape(48, 512)
    assert same_bits_or_both_nan(W, d["W_q4"])
    E, N, K = gg.shape("blk.0.ffn_gate_exps.weight")
    assert (E, N, K) == (4, 32, 512) and gg.type_name("blk.0.ffn_gate_exps.weight") == "Q6_K"
    raw = gg.raw("blk.0.ffn_gate_exps.weight")
    per = formats.gguf_tensor_nbytes(14, N * K)
    for e in range(E):
        We = ogg.dequant("Q6_K", bytes(raw[e * per:(e + 1) * per]), N * K).reshape(N, K)
        assert same_bits_or_both_nan(We, d["W_q6"][e])
    gg.close()


def test_gguf_rejects_non_gguf(tmp_path):
    p = tmp_path / "x.bin"
    p.write_bytes(b"\0" * 64)
    with pytest.raises(ValueError):
        formats.GGUFFile(str(p))


def test_safetensors_round_trip(tmp_path):
    rng = np.random.default_rng(0)
    t = {"a.qweight": rng.integers(-2 ** 31, 2 ** 31 - 1, (16, 24), dtype=np.int64).astype(np.int32),
         "a.scales": rng.standard_normal((2, 24)).astype(np.float16),
         "b": rng.standard_normal((3, 5)).astype(np.float32),
         "c": torch.randn(4, 6).to(torch.bfloat16)}
    p = str(tmp_path / "model.safetensors")
    formats.write_safetensors(p, t, metadata={"format": "pt"})
    st = formats.SafeTensors(p)
    assert st.metadata == {"format": "pt"}
    assert st.info("a.qweight") == ("I32", (16, 24)) and st.info("c") == ("BF16", (4, 6))
    assert np.array_equal(st.numpy("a.qweight"), t["a.qweight"])
    assert np.array_equal(st.numpy("a.scales").view(np.uint16), t["a.scales"].view(np.uint16))
    assert np.array_equal(st.numpy("b"), t["b"])
    # BF16 widens to fp32 exactly (a 16-bit shift, llm.py:556-557)
    assert np.array_equal(st.numpy("c"), t["c"].float().numpy())
    st.close()


def test_sharded_checkpoint_and_config(tmp_path):
    rng = np.random.default_rng(1)
    a = {"l0.qweight": rng.integers(0, 9, (4, 8)).astype(np.int32)}
    b = {"l1.qweight": rng.integers(0, 9, (4, 8)).astype(np.int32)}
    formats.write_safetensors(str(tmp_path / "model-00001.safetensors"), a)
    formats.write_safetensors(str(tmp_path / "model-00002.safetensors"), b)
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps(
        {"weight_map": {"l0.qweight": "model-00001.safetensors", "l1.qweight": "model-00002.safetensors"}}))
    (tmp_path / "config.json").write_text(json.dumps(
        {"quantization_config": {"bits": 4, "group_size": 128, "desc_act": True}}))
    d = formats.SafeTensorsDir(str(tmp_path))
    assert "l0.qweight" in d and "l1.qweight" in d and "l2.qweight" not in d
    assert np.array_equal(d.numpy("l1.qweight"), b["l1.qweight"])
    assert formats.autogptq_config(d.config()) == (128, 4, True)


def test_tensor_nbytes():
    assert formats.gguf_tensor_nbytes(12, 4096) == 16 * 144
    assert formats.gguf_tensor_nbytes(8, 64) == 2 * 34
    with pytest.raises(ValueError):
        formats.gguf_tensor_nbytes(14, 100)
