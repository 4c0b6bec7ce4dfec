"""Generate the golden fixtures in this folder by running the REFERENCE's own CPU code.

Run in a container where the reference project (xnetsc/webpytorch) is importable:
    python tests/golden/make_golden.py [path-to-reference-checkout]
It imports `webtorch` from that checkout (no cupy there, so `_core.GPU` is False and every
operator takes its numpy path), runs the qlinear / Q4_K / MoE paths on seeded inputs and
saves inputs and outputs as .npz files here. Tests never import the reference; they read
these files, which is what lets them run on a machine without it.

Cases:
  gptq_ref_*.npz   the reference's own correctness shapes (examples/gptq_int4_correctness.py:30-37):
                   weights from the reference quantiser `_gptq_quantize`, zero offset 0,
                   M in {1, 3, 4, 5, 32}; outputs of `QuantizedLinear(...)(Tensor(x))`.
  gptq_autogptq_*.npz  synthetic AutoGPTQ tensors through `QuantizedLinear.from_autogptq`
                   (zero offset 1), including the config-0 shape (K=896, N=4864, M=1) and int8.
  gptq_fromlinear.npz  `QuantizedLinear.from_linear` with K/N padding and a bias.
  q4k_*.npz        raw Q4_K bytes, `ggufload.dequant` output and x @ W.T.
  moe_*.npz        `lm_engine.moe_mlp` with a stub router returning fixed logits and
                   `QuantizedLinear.from_autogptq` experts.
  ggml_<type>_*.npz  raw Q8_0 / Q5_K / Q6_K bytes (benchmark-like and unrestricted random),
                   `ggufload.dequant` output and x @ W.T.
  gptq_writer_*.npz  the AutoGPTQ writer: `quantize._quantize_raw` + `_pack_autogptq` on a
                   padded (out, in) weight (qweight, qzeros storing zp - 1, fp16 scales, g_idx).
  gguf_parse.npz   a small GGUF file (metadata of every value type, a 2-D Q4_K weight, a stacked
                   Q6_K expert tensor, an F32 norm) and `ggufload.parse_header`'s view of it.
"""
import json
import struct
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from webpytorch_b200 import synth  # noqa: E402  (seeded generators shared with bench.py)


def _import_reference(path):
    sys.path.insert(0, path)
    from webtorch import _core as wt  # noqa
    from webtorch import ggufload as G  # noqa
    from webtorch import lm_engine as LE  # noqa
    from webtorch import quantize as Q  # noqa
    assert not wt.GPU, "the reference must run its numpy path here"
    return wt, G, LE, Q


def gptq_ref_cases(wt):
    rng = np.random.default_rng(0)
    for (K, N, gs, bits) in [(128, 64, 32, 4), (256, 128, 128, 4), (512, 256, 128, 4),
                             (128, 24, 32, 4), (256, 64, 32, 8), (384, 128, 128, 8)]:
        W = (rng.standard_normal((K, N)) * 0.1).astype(np.float32)
        qw, qz, sc, _, _ = wt._gptq_quantize(W, gs, bits)
        ql = wt.QuantizedLinear(qw, qz, sc, np.zeros((N,), np.float32), K, N, K, N, gs, bits)
        d = {"K": K, "N": N, "gs": gs, "bits": bits, "zoff": 0.0, "qweight": qw, "qzeros": qz,
             "scales": sc}
        # the exact weight the reference forms inside _gptq_matmul_np (_core.py:4069)
        per = 32 // bits
        q = np.empty((K, N), np.int32)
        for r in range(per):
            q[r::per] = (qw >> (bits * r)) & ((1 << bits) - 1)
        z = np.empty((K // gs, N), np.int32)
        for r in range(per):
            z[:, r::per] = (qz >> (bits * r)) & ((1 << bits) - 1)
        g = np.arange(K) // gs
        d["W"] = (sc[g] * (q - (z[g] + 0.0))).astype(np.float32)
        for M in (1, 3, 4, 5, 32):
            x = (rng.standard_normal((M, K)) * 0.5).astype(np.float32)
            d["x_%d" % M] = x
            d["y_%d" % M] = ql(wt.Tensor(x)).numpy()
        np.savez_compressed(os.path.join(HERE, "gptq_ref_K%d_N%d_g%d_b%d.npz" % (K, N, gs, bits)), **d)


def gptq_autogptq_cases(wt):
    for (K, N, gs, bits, M, seed, with_bias) in [(896, 4864, 128, 4, 1, 0, False),
                                                 (256, 128, 128, 8, 5, 1, True),
                                                 (512, 192, 128, 4, 16, 2, True),
                                                 (256, 96, 32, 4, 3, 3, False)]:
        rng = np.random.default_rng(seed)
        w = synth.gptq_weights(K, N, bits, gs, rng=rng)
        x = rng.standard_normal((M, K)).astype(np.float16)
        bias = rng.standard_normal(N).astype(np.float32) if with_bias else None
        ql = wt.QuantizedLinear.from_autogptq(w["qweight"], w["qzeros"], w["scales"], bias, gs, bits)
        y = ql(wt.Tensor(x.astype(np.float32))).numpy()
        d = {"K": K, "N": N, "gs": gs, "bits": bits, "zoff": 1.0, "x": x, "y": y,
             "qweight": w["qweight"], "qzeros": w["qzeros"], "scales": w["scales"]}
        if bias is not None:
            d["bias"] = bias
        np.savez_compressed(os.path.join(HERE, "gptq_autogptq_K%d_N%d_g%d_b%d.npz" % (K, N, gs, bits)), **d)


def gptq_fromlinear_case(wt):
    rng = np.random.default_rng(7)
    K, N, gs, bits = 200, 60, 32, 4
    lin = wt.Linear(K, N)
    lin.weight.data[...] = (rng.standard_normal((K, N)) * 0.1).astype(np.float32)
    lin.bias.data[...] = rng.standard_normal(N).astype(np.float32)
    ql = wt.QuantizedLinear.from_linear(lin, group_size=gs, bits=bits)
    x = (rng.standard_normal((2, 3, K)) * 0.5).astype(np.float32)
    y = ql(wt.Tensor(x)).numpy()
    np.savez_compressed(os.path.join(HERE, "gptq_fromlinear.npz"), K=K, N=N, gs=gs, bits=bits,
                        Kp=ql.Kp, Np=ql.Np, weight=np.asarray(lin.weight.data), bias=np.asarray(lin.bias.data),
                        qweight=np.asarray(ql.qweight), qzeros=np.asarray(ql.qzeros),
                        scales=np.asarray(ql.scales), x=x, y=y)


def q4k_cases(G):
    # (a) the reference self-check's recipe (_core.py:3697-3705): two random-byte blocks, redrawn
    # until the dequantised values are finite and below 1e4
    for seed in range(1000):
        rng = np.random.default_rng(seed)
        raw = rng.integers(0, 256, (2, 144), dtype=np.uint8)
        W = np.asarray(G.dequant(12, raw.tobytes(), 2 * 256), np.float32).reshape(2, 256)
        if np.all(np.isfinite(W)) and float(np.abs(W).max()) < 1e4:
            break
    else:
        raise RuntimeError("no finite random Q4_K block found")
    x = rng.standard_normal((3, 256)).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "q4k_randombytes.npz"), N=2, K=256, raw=raw, W=W, x=x,
                        y=(x @ W.T).astype(np.float32), seed=seed)
    # (a') unrestricted random bytes (inf / nan scales included): the decode must agree bit for bit
    # on every non-NaN value and put NaNs in the same places
    rng = np.random.default_rng(12345)
    raw = rng.integers(0, 256, (8, 2 * 144), dtype=np.uint8)
    W = np.asarray(G.dequant(12, raw.tobytes(), 8 * 512), np.float32).reshape(8, 512)
    np.savez_compressed(os.path.join(HERE, "q4k_rawbytes_nonfinite.npz"), N=8, K=512, raw=raw, W=W)
    # (b) the benchmark distribution (config 2) at a small size
    rng = np.random.default_rng(11)
    N, K = 64, 1024
    raw = synth.q4k_weights(N, K, rng=rng)
    W = np.asarray(G.dequant(12, raw.tobytes(), N * K), np.float32).reshape(N, K)
    d = {"N": N, "K": K, "raw": raw, "W": W}
    for M in (1, 8, 13):
        x = rng.standard_normal((M, K)).astype(np.float32)
        d["x_%d" % M] = x
        d["y_%d" % M] = (x @ W.T).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "q4k_synth.npz"), **d)


def moe_cases(wt, LE):
    for (E, top_k, H, I, T, seed) in [(8, 2, 128, 64, 5, 0), (16, 8, 256, 128, 12, 1)]:
        rng = np.random.default_rng(100 + seed)
        exps = synth.moe_experts(E, H, I, bits=4, gs=64, rng=rng)
        logits = rng.standard_normal((T, E)).astype(np.float32)
        x = rng.standard_normal((T, H)).astype(np.float32)

        class _LM:
            pass
        lm = _LM()
        lm.H = H
        experts = [{k: wt.QuantizedLinear.from_autogptq(e[k]["qweight"], e[k]["qzeros"], e[k]["scales"],
                                                         None, 64, 4) for k in ("gate", "up", "down")}
                   for e in exps]
        lay = {"moe": {"gate": (lambda t, _l=logits: wt.Tensor(_l)), "top_k": top_k,
                       "norm_topk_prob": True, "experts": experts, "shared": None}}
        y = LE.moe_mlp(lm, lay, wt.Tensor(x)).numpy()
        d = {"E": E, "top_k": top_k, "H": H, "I": I, "T": T, "gs": 64, "bits": 4, "logits": logits, "x": x,
             "y": y}
        for i, e in enumerate(exps):
            for k in ("gate", "up", "down"):
                for f in ("qweight", "qzeros", "scales"):
                    d["e%d_%s_%s" % (i, k, f)] = e[k][f]
        np.savez_compressed(os.path.join(HERE, "moe_E%d_k%d_T%d.npz" % (E, top_k, T)), **d)


def moe_shared_case(wt, LE):
    """Qwen-style block: routed experts plus a shared expert gated by sigmoid(x @ g)."""
    E, top_k, H, I, T, SI = 4, 2, 128, 64, 6, 128
    rng = np.random.default_rng(300)
    exps = synth.moe_experts(E, H, I, bits=4, gs=64, rng=rng)
    sh = synth.moe_experts(1, H, SI, bits=4, gs=64, rng=rng)[0]
    logits = rng.standard_normal((T, E)).astype(np.float32)
    x = rng.standard_normal((T, H)).astype(np.float32)
    gate_w = (rng.standard_normal((H, 1)) * 0.05).astype(np.float32)

    class _LM:
        pass
    lm = _LM()
    lm.H = H

    def q(w):
        return wt.QuantizedLinear.from_autogptq(w["qweight"], w["qzeros"], w["scales"], None, 64, 4)
    experts = [{k: q(e[k]) for k in ("gate", "up", "down")} for e in exps]
    shared = {k: q(sh[k]) for k in ("gate", "up", "down")}
    lay = {"moe": {"gate": (lambda t, _l=logits: wt.Tensor(_l)), "top_k": top_k, "norm_topk_prob": False,
                   "experts": experts, "shared": shared,
                   "shared_gate": (lambda t: wt.Tensor(np.asarray(t.numpy(), np.float32) @ gate_w))}}
    y = LE.moe_mlp(lm, lay, wt.Tensor(x)).numpy()
    d = {"E": E, "top_k": top_k, "H": H, "I": I, "SI": SI, "T": T, "gs": 64, "bits": 4, "logits": logits,
         "x": x, "y": y, "shared_gate_w": gate_w, "norm_topk_prob": 0}
    for i, e in enumerate(exps):
        for k in ("gate", "up", "down"):
            for f in ("qweight", "qzeros", "scales"):
                d["e%d_%s_%s" % (i, k, f)] = e[k][f]
    for k in ("gate", "up", "down"):
        for f in ("qweight", "qzeros", "scales"):
            d["shared_%s_%s" % (k, f)] = sh[k][f]
    np.savez_compressed(os.path.join(HERE, "moe_shared_E%d_k%d_T%d.npz" % (E, top_k, T)), **d)


def ggml_kquant_cases(G):
    ids = {"Q8_0": 8, "Q5_K": 13, "Q6_K": 14}
    for t, tid in ids.items():
        rng = np.random.default_rng(tid)
        N, K = 64, 1024
        raw = synth.ggml_weights(t, N, K, rng=rng)
        W = np.asarray(G.dequant(tid, raw.tobytes(), N * K), np.float32).reshape(N, K)
        d = {"N": N, "K": K, "raw": raw, "W": W, "type_id": tid}
        for M in (1, 3, 8):
            x = rng.standard_normal((M, K)).astype(np.float32)
            d["x_%d" % M] = x
            d["y_%d" % M] = (x @ W.T).astype(np.float32)
        np.savez_compressed(os.path.join(HERE, "ggml_%s_synth.npz" % t), **d)
        # unrestricted random bytes (inf / nan scales included)
        vals, nbytes = (32, 34) if t == "Q8_0" else (256, {"Q5_K": 176, "Q6_K": 210}[t])
        raw = rng.integers(0, 256, (8, (512 // vals) * nbytes), dtype=np.uint8)
        W = np.asarray(G.dequant(tid, raw.tobytes(), 8 * 512), np.float32).reshape(8, 512)
        np.savez_compressed(os.path.join(HERE, "ggml_%s_rawbytes.npz" % t), N=8, K=512, raw=raw, W=W, type_id=tid)


def gptq_writer_cases(Q):
    for (N, K, gs, bits, seed) in [(100, 200, 64, 4, 0), (64, 256, 128, 8, 1), (480, 896, 128, 4, 2)]:
        rng = np.random.default_rng(seed)
        W = (rng.standard_normal((N, K)) * 0.05).astype(np.float16)
        W[0, :gs] = 0.25          # a group with one value: s = 0 -> 1e-8
        q, sc, zp, K_, N_, Kp, Np = Q._quantize_raw(W, gs, bits)
        qw, qz, scq, gidx = Q._pack_autogptq(q, sc, zp, gs, bits)
        np.savez_compressed(os.path.join(HERE, "gptq_writer_N%d_K%d_g%d_b%d.npz" % (N, K, gs, bits)), W=W, N=N, K=K,
                            gs=gs, bits=bits, Kp=Kp, Np=Np, qweight=qw, qzeros=qz, scales=scq, g_idx=gidx)


def _gguf_bytes(meta, tensors, align=32):
    """A GGUF v3 file: header, metadata KV, tensor infos, aligned data (test-fixture builder)."""
    def s_(x):
        b = x.encode()
        return struct.pack("<Q", len(b)) + b

    def val(t, v):
        fmt = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}
        if t == 8:
            return s_(v)
        if t == 9:
            at, items = v
            return struct.pack("<IQ", at, len(items)) + b"".join(val(at, i) for i in items)
        return struct.pack(fmt[t], v)
    out = struct.pack("<IIQQ", 0x46554747, 3, len(tensors), len(meta))
    for k, (t, v) in meta.items():
        out += s_(k) + struct.pack("<I", t) + val(t, v)
    off, data = 0, b""
    for name, dims, ttype, raw in tensors:
        pad = (-off) % align
        data += b"\0" * pad
        off += pad
        out += s_(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims) + \
            struct.pack("<IQ", ttype, off)
        data += raw
        off += len(raw)
    out += b"\0" * ((-len(out)) % align)
    return out + data


def gguf_parse_case(G):
    rng = np.random.default_rng(7)
    q4 = synth.q4k_weights(48, 512, rng=rng)                  # [out 48, in 512]
    q6 = synth.ggml_weights("Q6_K", 4 * 32, 512, rng=rng)     # 4 experts x [out 32, in 512]
    norm = rng.standard_normal(512).astype(np.float32)
    meta = {"general.architecture": (8, "qwen3moe"), "general.alignment": (4, 32), "a.u8": (0, 7),
            "a.i8": (1, -3), "a.u16": (2, 500), "a.i16": (3, -500), "a.i32": (5, -70000), "a.f32": (6, 0.5),
            "a.bool": (7, True), "a.u64": (10, 2 ** 40), "a.i64": (11, -2 ** 40), "a.f64": (12, 0.25),
            "a.arr": (9, (5, [1, -2, 3])), "a.strs": (9, (8, ["x", "yz"]))}
    tensors = [("blk.0.attn_norm.weight", [512], 0, norm.tobytes()),
               ("blk.0.attn_q.weight", [512, 48], 12, q4.tobytes()),
               ("blk.0.ffn_gate_exps.weight", [512, 32, 4], 14, q6.tobytes())]
    buf = _gguf_bytes(meta, tensors)
    version, md, infos, data_start = G.parse_header(buf)
    names = [t["name"] for t in infos]
    np.savez_compressed(os.path.join(HERE, "gguf_parse.npz"), gguf=np.frombuffer(buf, np.uint8), version=version,
                        meta=json.dumps(md), names=json.dumps(names),
                        dims=json.dumps([[int(d) for d in t["dims"]] for t in infos]),
                        types=np.array([t["type"] for t in infos], np.int32),
                        offsets=np.array([t["offset"] for t in infos], np.int64), data_start=data_start,
                        W_q4=np.asarray(G.dequant(12, q4.tobytes(), 48 * 512), np.float32).reshape(48, 512),
                        W_q6=np.asarray(G.dequant(14, q6.tobytes(), 128 * 512), np.float32).reshape(4, 32, 512),
                        norm=norm)


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("WEBTORCH_REFERENCE")
    if not ref:
        sys.exit("usage: make_golden.py <reference checkout> (or set WEBTORCH_REFERENCE)")
    wt, G, LE, Q = _import_reference(ref)
    gptq_ref_cases(wt)
    gptq_autogptq_cases(wt)
    gptq_fromlinear_case(wt)
    q4k_cases(G)
    moe_cases(wt, LE)
    moe_shared_case(wt, LE)
    ggml_kquant_cases(G)
    gptq_writer_cases(Q)
    gguf_parse_case(G)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
