"""GPTQ oracle (numpy) — test infrastructure, restating the reference's CPU path.

All arithmetic follows webtorch/_core.py:4046-4072 exactly: values are unpacked LSB-first,
`w = (sc[g] * (q - (z[g] + zoff))).astype(float32)` is formed in float64 and rounded once,
and the product is `x @ w` in float32 per 2048-column block.
"""
import numpy as np


def unpack_rows(qweight, bits):
    """q[k, n] from qweight [K/per, N] packed LSB-first along K (_core.py:4061-4063)."""
    qw = np.asarray(qweight, np.int32)
    per = 32 // bits
    qmax = (1 << bits) - 1
    q = np.empty((qw.shape[0] * per, qw.shape[1]), np.int32)
    for r in range(per):
        q[r::per] = (qw >> (bits * r)) & qmax
    return q


def unpack_cols(qzeros, bits):
    """z[g, n] from qzeros [G, N/per] packed LSB-first along N (_core.py:4065-4067)."""
    qz = np.asarray(qzeros, np.int32)
    per = 32 // bits
    qmax = (1 << bits) - 1
    z = np.empty((qz.shape[0], qz.shape[1] * per), np.int32)
    for r in range(per):
        z[:, r::per] = (qz >> (bits * r)) & qmax
    return z


def group_index(K, gs, g_idx=None):
    """Group of every contracted row: arange(K)//gs in the reference (_core.py:4056); the
    desc_act restatement uses the checkpoint's g_idx instead."""
    return np.arange(K) // gs if g_idx is None else np.asarray(g_idx, np.int64)


def gptq_dequant(qweight, qzeros, scales, gs, bits, zoff=0.0, g_idx=None):
    """Exact fp32 [K, N] weight, following _core.py:4060-4069 (float64 then one rounding)."""
    q = unpack_rows(qweight, bits)
    z = unpack_cols(qzeros, bits)
    sc = np.asarray(scales, np.float32)
    g = group_index(q.shape[0], gs, g_idx)
    return (sc[g] * (q - (z[g] + zoff))).astype(np.float32)


def gptq_matmul(xf, qweight, qzeros, scales, K, N, gs, bits, zoff=0.0, g_idx=None, block=2048):
    """Restates `_gptq_matmul_np` (_core.py:4046-4072); `g_idx` generalises line 4056."""
    x = np.asarray(xf, np.float32)
    qw = np.asarray(qweight)
    qz = np.asarray(qzeros)
    sc = np.asarray(scales, np.float32)
    per = 32 // bits
    qmax = (1 << bits) - 1
    Kp = int(qw.shape[0]) * per
    g = group_index(Kp, gs, g_idx)
    out = np.empty((int(x.shape[0]), N), np.float32)
    z_full = unpack_cols(qz, bits)
    for c0 in range(0, N, block):
        c1 = min(N, c0 + block)
        qwb = qw[:, c0:c1]
        q = np.empty((Kp, c1 - c0), np.int32)
        for r in range(per):
            q[r::per] = (qwb >> (bits * r)) & qmax
        z = z_full[:, c0:c1]
        w = (sc[g, c0:c1] * (q - (z[g] + zoff))).astype(np.float32)
        out[:, c0:c1] = x @ w
    return out


def gptq_matmul_np_steps(xf, qweight, qzeros, scales, K, N, gs, bits, zoff=0.0, block=2048):
    """`_gptq_matmul_np` (webtorch/_core.py:4046-4072) statement for statement, for timing.

    Unlike `gptq_matmul` above (which unpacks the zero points once), this keeps every step of
    the reference, including the unpack of ALL of qzeros inside every 2048-column block
    (_core.py:4065-4068), so a CPU timing of it measures the reference's own work."""
    x = np.asarray(xf, np.float32)
    qw = np.asarray(qweight)
    qz = np.asarray(qzeros)
    sc = np.asarray(scales, np.float32)
    per = 32 // bits
    qmax = (1 << bits) - 1
    Kp = int(qw.shape[0]) * per
    g = np.arange(Kp) // gs
    out = np.empty((int(x.shape[0]), N), np.float32)
    for c0 in range(0, N, block):
        c1 = min(N, c0 + block)
        qwb = qw[:, c0:c1]
        q = np.empty((Kp, c1 - c0), np.int32)
        for r in range(per):
            q[r::per] = (qwb >> (bits * r)) & qmax
        z_full = np.empty((int(qz.shape[0]), N), np.int32)
        for r in range(per):
            z_full[:, r::per] = (qz >> (bits * r)) & qmax
        z = z_full[:, c0:c1]
        del z_full
        w = (sc[g, c0:c1] * (q - (z[g] + zoff))).astype(np.float32)
        out[:, c0:c1] = x @ w
        del q, z, w
    return out


def quantized_linear(x, qweight, qzeros, scales, bias, K, N, Kp, Np, gs, bits, zoff, g_idx=None):
    """`QuantizedLinear.forward` (_core.py:4446-4456): pad K, matmul, slice N, add bias."""
    xd = np.asarray(x, np.float32)
    lead = xd.shape[:-1]
    xf = xd.reshape(-1, K)
    if Kp != K:
        xp_ = np.zeros((xf.shape[0], Kp), np.float32)
        xp_[:, :K] = xf
        xf = xp_
    of = gptq_matmul(xf, qweight, qzeros, scales, Kp, Np, gs, bits, zoff, g_idx)
    if Np != N:
        of = np.ascontiguousarray(of[:, :N])
    b = np.zeros((N,), np.float32) if bias is None else np.asarray(bias, np.float32)
    return (of + b).reshape(*lead, N)


def gptq_quantize(W, group_size=32, bits=4):
    """Asymmetric min/max quantiser and packer, restating _core.py:3782-3824 (zero offset 0).

    Arithmetic runs in W's own float dtype (the reference's `Linear` holds float64 weights,
    _core.py:474), and scales are stored as float32, as in the reference."""
    W = np.asarray(W)
    if W.dtype not in (np.float32, np.float64):
        W = W.astype(np.float32)
    K, N = W.shape
    per = 32 // bits
    qmax = (1 << bits) - 1
    assert K % group_size == 0 and K % per == 0 and N % per == 0
    nG = K // group_size
    scales = np.zeros((nG, N), np.float32)
    zeros = np.zeros((nG, N), np.int32)
    q = np.empty((K, N), np.int32)
    for g in range(nG):
        blk = W[g * group_size:(g + 1) * group_size]
        wmin = blk.min(0)
        wmax = blk.max(0)
        sc = (wmax - wmin) / qmax
        sc[sc == 0] = 1e-8
        zp = np.clip(np.round(-wmin / sc), 0, qmax).astype(np.int32)
        scales[g] = sc
        zeros[g] = zp
        q[g * group_size:(g + 1) * group_size] = np.clip(np.round(blk / sc) + zp, 0, qmax).astype(np.int32)
    return pack_rows(q, bits), pack_cols(zeros, bits), scales, K, N


def pack_rows(q, bits):
    """Pack [K, N] values LSB-first along K into int32 [K/per, N] (_core.py:3815-3819)."""
    q = np.asarray(q, np.int64)
    per = 32 // bits
    acc = np.zeros((q.shape[0] // per, q.shape[1]), np.int64)
    for j in range(per):
        acc |= (q[j::per] & ((1 << bits) - 1)) << (bits * j)
    return acc.astype(np.uint32).view(np.int32)


def pack_cols(z, bits):
    """Pack [G, N] values LSB-first along N into int32 [G, N/per] (_core.py:3821-3822)."""
    z = np.asarray(z, np.int64)
    per = 32 // bits
    acc = np.zeros((z.shape[0], z.shape[1] // per), np.int64)
    for j in range(per):
        acc |= (z[:, j::per] & ((1 << bits) - 1)) << (bits * j)
    return acc.astype(np.uint32).view(np.int32)


def pack_autogptq(q, sc, zp, gs, bits):
    """AutoGPTQ writer (quantize.py:96-106): stores (zp - 1) & mask, fp16 scales, g_idx = k//gs."""
    Kp = q.shape[0]
    zpm = (np.asarray(zp, np.int64) - 1) & ((1 << bits) - 1)
    return pack_rows(q, bits), pack_cols(zpm, bits), np.asarray(sc).astype(np.float16), \
        (np.arange(Kp, dtype=np.int32) // gs)


def sort_rows(qweight, perm, bits):
    """Row k' of the result holds value perm[k'] of qweight (loader-side desc_act sort)."""
    return pack_rows(unpack_rows(qweight, bits)[np.asarray(perm)], bits)


def quantize_raw(W_out_in, gs, bits):
    """The AutoGPTQ writer's quantiser, webtorch/quantize.py:80-95 (`_quantize_raw`): the (out, in)
    weight in float32, transposed to (K, N), zero-padded to Kp (multiple of gs) and Np (multiple
    of per); returns q [Kp, Np], scales [Kp/gs, Np] float32, zero points [Kp/gs, Np]."""
    Wt = np.ascontiguousarray(np.asarray(W_out_in, np.float32).T)
    K, N = Wt.shape
    qmax = (1 << bits) - 1
    per = 32 // bits
    Kp = K + ((-K) % gs)
    Np = N + ((-N) % per)
    if Kp != K or Np != N:
        Wt = np.pad(Wt, ((0, Kp - K), (0, Np - N)))
    nG = Kp // gs
    sc = np.empty((nG, Np), np.float32)
    zp = np.empty((nG, Np), np.int32)
    q = np.empty((Kp, Np), np.int32)
    for g in range(nG):
        blk = Wt[g * gs:(g + 1) * gs]
        lo = blk.min(0)
        hi = blk.max(0)
        s = (hi - lo) / qmax
        s[s == 0] = 1e-8
        z = np.clip(np.round(-lo / s), 0, qmax).astype(np.int32)
        sc[g] = s
        zp[g] = z
        q[g * gs:(g + 1) * gs] = np.clip(np.round(blk / s) + z, 0, qmax).astype(np.int32)
    return q, sc, zp
