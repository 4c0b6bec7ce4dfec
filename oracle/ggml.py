"""GGUF Q8_0 / Q5_K / Q6_K oracle (numpy) — test infrastructure, restating the reference's
dequantiser branches of webtorch/ggufload.py:140-145 (Q8_0), 210-246 (Q6_K, Q5_K), value for
value in float32, and GGMLLinear.forward (webtorch/_core.py:4399-4406) as x @ W.T.
"""
import numpy as np

from .q4k import dequant as q4k_dequant


def _f16(b):
    return np.ascontiguousarray(b).view(np.float16).astype(np.float32)


def _scales_k4(s):
    """get_scale_min_k4 on (blk, 12) bytes -> sc, m (blk, 8) float32 (ggufload.py:120-131)."""
    sc = np.empty((s.shape[0], 8), np.float32)
    m = np.empty((s.shape[0], 8), np.float32)
    for j in range(8):
        if j < 4:
            sc[:, j] = s[:, j] & 63
            m[:, j] = s[:, j + 4] & 63
        else:
            sc[:, j] = (s[:, j + 4] & 0x0F) | ((s[:, j - 4] >> 6) << 4)
            m[:, j] = (s[:, j + 4] >> 4) | ((s[:, j] >> 6) << 4)
    return sc, m


def dequant(type_name, raw, n):
    """fp32 values of n weights of a ggml type (row-major, ggml order)."""
    u8 = np.frombuffer(bytes(raw), np.uint8)
    if type_name == "Q4_K":
        return q4k_dequant(raw, n)
    if type_name == "Q8_0":                        # ggufload.py:140-145
        blk = n // 32
        b = u8[:blk * 34].reshape(blk, 34)
        return (_f16(b[:, :2]) * b[:, 2:].view(np.int8).astype(np.float32)).reshape(-1)[:n]
    if type_name == "Q6_K":                        # ggufload.py:210-229
        blk = n // 256
        b = u8[:blk * 210].reshape(blk, 210)
        ql, qh = b[:, 0:128], b[:, 128:192]
        sc = b[:, 192:208].view(np.int8).astype(np.float32)
        d = _f16(b[:, 208:210])
        out = np.empty((blk, 256), np.float32)
        for h in range(2):
            qlh, qhh, sch = ql[:, 64 * h:64 * (h + 1)], qh[:, 32 * h:32 * (h + 1)], sc[:, 8 * h:8 * (h + 1)]
            for l in range(32):
                ii = l // 16
                for t in range(4):
                    lo = qlh[:, l + 32 * (t & 1)]
                    nib = (lo >> 4) if t >= 2 else (lo & 0x0F)
                    q = (nib | (((qhh[:, l] >> (2 * t)) & 3) << 4)).astype(np.int16) - 32
                    out[:, 128 * h + 32 * t + l] = d[:, 0] * sch[:, ii + 2 * t] * q
        return out.reshape(-1)[:n]
    if type_name == "Q5_K":                        # ggufload.py:230-246
        blk = n // 256
        b = u8[:blk * 176].reshape(blk, 176)
        d, dmin = _f16(b[:, 0:2]), _f16(b[:, 2:4])
        sc, m = _scales_k4(b[:, 4:16])
        qh, qs = b[:, 16:48], b[:, 48:176]
        out = np.empty((blk, 256), np.float32)
        for g in range(4):
            ql = qs[:, 32 * g:32 * (g + 1)]
            i0 = 2 * g
            lo = (ql & 0x0F).astype(np.float32) + np.where(qh & np.uint8(1 << i0), 16.0, 0.0)
            hi = (ql >> 4).astype(np.float32) + np.where(qh & np.uint8(1 << (i0 + 1)), 16.0, 0.0)
            out[:, 32 * i0:32 * (i0 + 1)] = d * sc[:, i0:i0 + 1] * lo - dmin * m[:, i0:i0 + 1]
            out[:, 32 * (i0 + 1):32 * (i0 + 2)] = d * sc[:, i0 + 1:i0 + 2] * hi - dmin * m[:, i0 + 1:i0 + 2]
        return out.reshape(-1)[:n]
    raise NotImplementedError(type_name)


def matmul(x, raw, type_name, K, N, bias=None):
    """GGMLLinear.forward semantics: x[M, K] @ W[N, K].T (+ bias) in float32."""
    W = dequant(type_name, raw, N * K).reshape(N, K)
    y = np.asarray(x, np.float32) @ W.T
    if bias is not None:
        y = y + np.asarray(bias, np.float32)
    return y.astype(np.float32)
