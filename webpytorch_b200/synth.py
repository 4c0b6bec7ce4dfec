"""Seeded synthetic tensors with the shapes and value distributions of the benchmark configs.

No checkpoints are available offline, so these stand in for them (numpy default_rng(seed)):
  * GPTQ (configs 0, 1, 3): qweight int32 [K/per, N] of uniform 32-bit words (every packed
    value uniform), scales fp16 U[0.002, 0.02] [K/gs, N], qzeros int32 [K/gs, N/per] of
    uniform packed values, g_idx = arange(K)//gs, or for desc_act a random permutation of it.
  * Q4_K (config 2): super-blocks with fp16 d, dmin U[1e-3, 1e-2], eight 6-bit scales and
    mins uniform on 0..63 packed as get_scale_min_k4 reads them, 128 uniform nibble bytes.
  * MoE (config 4): router logits N(0, 1) [T, E]; experts as GPTQ int4 g128 weights.
"""
import numpy as np


def gptq_weights(K, N, bits=4, gs=128, seed=0, desc_act=False, rng=None):
    """Returns dict(qweight, qzeros, scales(fp16), g_idx) as numpy arrays."""
    rng = rng if rng is not None else np.random.default_rng(seed)
    per = 32 // bits
    G = K // gs
    qweight = rng.integers(0, 2 ** 32, size=(K // per, N), dtype=np.uint64).astype(np.uint32).view(np.int32)
    scales = rng.uniform(0.002, 0.02, size=(G, N)).astype(np.float16)
    qzeros = rng.integers(0, 2 ** 32, size=(G, N // per), dtype=np.uint64).astype(np.uint32).view(np.int32)
    g_idx = (np.arange(K) // gs).astype(np.int32)
    if desc_act:
        g_idx = g_idx[rng.permutation(K)].astype(np.int32)
    return {"qweight": qweight, "qzeros": qzeros, "scales": scales, "g_idx": g_idx}


def pack_q4k_scales(sc, m):
    """Inverse of get_scale_min_k4: (blk, 8) 6-bit scales and mins -> (blk, 12) bytes."""
    sc = np.asarray(sc, np.uint8)
    m = np.asarray(m, np.uint8)
    s = np.zeros((sc.shape[0], 12), np.uint8)
    s[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
    s[:, 4:8] = (m[:, 0:4] & 63) | ((m[:, 4:8] >> 4) << 6)
    s[:, 8:12] = (sc[:, 4:8] & 0x0F) | ((m[:, 4:8] & 0x0F) << 4)
    return s


def q4k_weights(N, K, seed=0, rng=None):
    """Raw Q4_K bytes for a [N, K] weight (rows along N, 256-value blocks along K): uint8 [N, K/256*144]."""
    rng = rng if rng is not None else np.random.default_rng(seed)
    assert K % 256 == 0
    nb = N * (K // 256)
    blk = np.empty((nb, 144), np.uint8)
    blk[:, 0:2] = rng.uniform(1e-3, 1e-2, size=(nb, 1)).astype(np.float16).view(np.uint8)
    blk[:, 2:4] = rng.uniform(1e-3, 1e-2, size=(nb, 1)).astype(np.float16).view(np.uint8)
    sc = rng.integers(0, 64, size=(nb, 8), dtype=np.uint8)
    mn = rng.integers(0, 64, size=(nb, 8), dtype=np.uint8)
    blk[:, 4:16] = pack_q4k_scales(sc, mn)
    blk[:, 16:144] = rng.integers(0, 256, size=(nb, 128), dtype=np.uint8)
    return blk.reshape(N, (K // 256) * 144)


def activations(M, K, dtype=np.float16, seed=0, rng=None):
    rng = rng if rng is not None else np.random.default_rng(seed)
    return rng.standard_normal((M, K)).astype(np.float32).astype(dtype)


def moe_experts(E, hidden, inter, bits=4, gs=128, seed=0, rng=None):
    """Per expert: gate/up [hidden -> inter] each and down [inter -> hidden] (GPTQ packs)."""
    rng = rng if rng is not None else np.random.default_rng(seed)
    out = []
    for _ in range(E):
        out.append({"gate": gptq_weights(hidden, inter, bits, gs, rng=rng),
                    "up": gptq_weights(hidden, inter, bits, gs, rng=rng),
                    "down": gptq_weights(inter, hidden, bits, gs, rng=rng)})
    return out


def ggml_weights(type_name, N, K, seed=0, rng=None):
    """Raw GGUF bytes [N, K/block * bytes] of a Q8_0, Q5_K or Q6_K weight: fp16 scales (d, dmin)
    uniform on [1e-3, 1e-2], every other byte uniform (6-bit scale/min fields as Q4_K's)."""
    rng = rng if rng is not None else np.random.default_rng(seed)
    if type_name == "Q4_K":
        return q4k_weights(N, K, rng=rng)
    vals, nbytes = {"Q8_0": (32, 34), "Q5_K": (256, 176), "Q6_K": (256, 210)}[type_name]
    assert K % vals == 0
    nb = N * (K // vals)
    blk = rng.integers(0, 256, size=(nb, nbytes), dtype=np.uint8)
    d = rng.uniform(1e-3, 1e-2, size=(nb, 2)).astype(np.float16).view(np.uint8).reshape(nb, 4)
    if type_name == "Q8_0":
        blk[:, 0:2] = d[:, 0:2]
    elif type_name == "Q5_K":
        blk[:, 0:4] = d
        sc = rng.integers(0, 64, size=(nb, 8), dtype=np.uint8)
        mn = rng.integers(0, 64, size=(nb, 8), dtype=np.uint8)
        blk[:, 4:16] = pack_q4k_scales(sc, mn)
    else:
        blk[:, 208:210] = d[:, 0:2]
    return blk.reshape(N, (K // vals) * nbytes)
