"""GGUF Q4_K oracle (numpy) — test infrastructure, restating webtorch/ggufload.py.

Block layout (256 values / 144 bytes): f16 d | f16 dmin | scales[12] | qs[128].
Sub-block j (32 values) has a 6-bit scale sc_j and min m_j (`get_scale_min_k4`,
ggufload.py:120-131); value = d*sc_j * q - dmin*m_j, q being the low nibbles of
qs[32g : 32g+32] for j = 2g and the high nibbles for j = 2g+1 (ggufload.py:190-202).
"""
import numpy as np

BLOCK_VALUES = 256
BLOCK_BYTES = 144


def _f16(u8_pairs):
    """(blk, 2) uint8 -> (blk, 1) float32 (ggufload.py:116-117)."""
    return np.ascontiguousarray(u8_pairs).view(np.float16).astype(np.float32)


def scale_min(s):
    """Eight 6-bit scales and mins from 12 bytes (ggufload.py:120-131)."""
    blk = s.shape[0]
    sc = np.empty((blk, 8), np.float32)
    m = np.empty((blk, 8), np.float32)
    for j in range(8):
        if j < 4:
            sc[:, j] = s[:, j] & 63
            m[:, j] = s[:, j + 4] & 63
        else:
            sc[:, j] = (s[:, j + 4] & 0x0F) | ((s[:, j - 4] >> 6) << 4)
            m[:, j] = (s[:, j + 4] >> 4) | ((s[:, j] >> 6) << 4)
    return sc, m


def dequant(raw, n):
    """First n values of a Q4_K byte stream as float32 (ggufload.py:190-202)."""
    u8 = np.frombuffer(raw, np.uint8) if isinstance(raw, (bytes, bytearray, memoryview)) else \
        np.asarray(raw, np.uint8).reshape(-1)
    blk = n // BLOCK_VALUES
    b = u8[:blk * BLOCK_BYTES].reshape(blk, BLOCK_BYTES)
    d = _f16(b[:, 0:2])
    dmin = _f16(b[:, 2:4])
    sc, m = scale_min(b[:, 4:16])
    qs = b[:, 16:144]
    out = np.empty((blk, BLOCK_VALUES), np.float32)
    for g in range(4):
        q = qs[:, g * 32:(g + 1) * 32]
        i0 = 2 * g
        d1 = d * sc[:, i0:i0 + 1]
        m1 = dmin * m[:, i0:i0 + 1]
        d2 = d * sc[:, i0 + 1:i0 + 2]
        m2 = dmin * m[:, i0 + 1:i0 + 2]
        out[:, i0 * 32:(i0 + 1) * 32] = d1 * (q & 0x0F).astype(np.float32) - m1
        out[:, (i0 + 1) * 32:(i0 + 2) * 32] = d2 * (q >> 4).astype(np.float32) - m2
    return out.reshape(-1)[:n]


def matmul(x, raw, K, N, bias=None):
    """GGMLLinear.forward semantics (webtorch/_core.py:4399-4406): x[M,K] @ W[N,K].T (+ bias),
    with W the reference dequantiser's output, in float32."""
    W = dequant(raw, N * K).reshape(N, K)
    y = np.asarray(x, np.float32) @ W.T
    if bias is not None:
        y = y + np.asarray(bias, np.float32)
    return y.astype(np.float32)
