"""The decode step around the quantized linear: one token through a stack of transformer layers
with the norms, SwiGLU and residuals fused into the GPTQ GEMVs, and the whole step captured in
one CUDA graph that is replayed for every token.

Reference counterparts (package `webtorch`): the layer math of lm_engine.py:62-107 (`_rms`,
`_rope`, `_rot`, `_mlp`, `_block`) and the capture-replay decode of llm.py:1573-1616
(`_set_inputs` writes the token's embedding and position into fixed buffers, `_decode_fwd` runs
the layers, the captured command list is replayed; llm.py:1796-1814). Per layer:

    x  = rms(h, in_ln)                 fused into the QKV GEMV's activation staging
    q, k, v = x @ Wqkv + b             one GEMV over the concatenated q | k | v weights
    q, k = rope(q), rope(k); cache k, v; o = softmax(q K^T / sqrt(HD)) V      (ql_decode_attention)
    h  = h + o @ Wo                    residual added in the O GEMV's epilogue
    x  = rms(h, post_ln)               fused into the gate | up GEMV
    h  = h + (silu(g) * u) @ Wdown     SwiGLU formed while the down GEMV stages [g | u]; residual

Five launches per layer, all of this library's kernels, chained by programmatic dependent launch
(each may start streaming its weights while the previous one finishes); buffers are fixed so the
step replays.
"""
import math

import numpy as np
import torch

from . import _ffi
from .qlinear import QuantizedLinear

__all__ = ["fused_linear", "concat_linears", "DecodeLayer", "DecodeStack", "rope_tables"]


def fused_linear(x, ql, *, norm_weight=None, norm_eps=1e-6, glu=0, residual=None, out=None, workspace=None,
                 stream=None):
    """out = prologue(x) @ W + bias (+ residual) for a QuantizedLinear `ql` (decode path, M <= 16):
    prologue = RMSNorm with `norm_weight` [K] fp32, or SwiGLU of [gate | up] rows when glu == K.
    `out` may be `residual` itself. Wraps ql_gptq_matmul_fused."""
    if ql.Kp != ql.Kt or ql.Np != ql.Nt:
        raise ValueError("fused_linear needs an unpadded QuantizedLinear (Kp == Kt, Np == Nt)")
    K, N = ql.Kp, ql.Np
    M = x.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=x.device)
    ws_bytes = workspace.numel() if workspace is not None else 0
    _ffi.call("ql_gptq_matmul_fused", x.data_ptr(), _ffi.dtype_code(x.dtype), x.stride(0), _ffi.ptr(ql.x_perm),
              ql.qweight.data_ptr(), ql.qzeros.data_ptr(), ql.scales.data_ptr(), _ffi.dtype_code(ql.scales.dtype),
              _ffi.ptr(ql.bias), _ffi.ptr(norm_weight), float(norm_eps), int(glu), _ffi.ptr(residual),
              residual.stride(0) if residual is not None else 0, out.data_ptr(), _ffi.dtype_code(out.dtype),
              out.stride(0), M, K, N, ql.gs, ql.bits, ql.zero_offset, _ffi.ptr(workspace), ws_bytes,
              _ffi.stream_ptr(stream, x.device))
    return out


def concat_linears(lins, device=None):
    """One QuantizedLinear computing [l0(x) | l1(x) | ...] (same K, group size, bits and zero
    offset): packed weights, zero points and scales concatenated along N (zero points are packed
    along N, so every N must be a multiple of 32 / bits). Used for q | k | v and gate | up."""
    l0 = lins[0]
    for l in lins:
        if (l.Kp, l.gs, l.bits, l.zero_offset) != (l0.Kp, l0.gs, l0.bits, l0.zero_offset) or l.x_perm is not None:
            raise ValueError("concat_linears: the linears must share K, group size, bits, zero offset, no act order")
    qw = torch.cat([l.qweight for l in lins], 1)
    qz = torch.cat([l.qzeros for l in lins], 1)
    sc = torch.cat([l.scales for l in lins], 1)
    Ns = [l.Np for l in lins]
    bias = None
    if any(l.bias is not None for l in lins):
        bias = torch.cat([l.bias if l.bias is not None else torch.zeros(l.Np, device=qw.device) for l in lins])
    return QuantizedLinear(qw, qz, sc, bias, l0.Kp, sum(Ns), l0.Kp, sum(Ns), l0.gs, l0.bits, l0.zero_offset,
                           device=device or qw.device)


def rope_tables(lmax, HD, theta):
    """cos / sin [lmax, HD/2] fp32, formed in float64 as lm_engine.py:66-70 does, then rounded."""
    inv = 1.0 / (theta ** (np.arange(0, HD, 2, dtype=np.float64) / HD))
    ang = np.arange(lmax, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


class DecodeLayer:
    """One layer's weights: q, k, v, o, gate, up, down QuantizedLinears (AutoGPTQ or reference
    packing) and the two RMSNorm weights [H]; q | k | v and gate | up are concatenated once."""

    def __init__(self, q, k, v, o, gate, up, down, in_ln, post_ln, device=None):
        dev = q.qweight.device if device is None else torch.device(device)
        self.qkv = concat_linears([q, k, v], dev)
        self.o = o
        self.gate_up = concat_linears([gate, up], dev)
        self.down = down
        self.in_ln = torch.as_tensor(np.asarray(in_ln, np.float32) if not isinstance(in_ln, torch.Tensor)
                                     else in_ln.float()).to(dev).contiguous()
        self.post_ln = torch.as_tensor(np.asarray(post_ln, np.float32) if not isinstance(post_ln, torch.Tensor)
                                       else post_ln.float()).to(dev).contiguous()
        self.I = down.Kp

    def nbytes(self):
        return self.qkv.nbytes() + self.o.nbytes() + self.gate_up.nbytes() + self.down.nbytes()


class DecodeStack:
    """A stack of DecodeLayers with fixed buffers, a KV cache and rotary tables. `step(embedding,
    pos)` runs one token: it writes the embedding and position into the step's input buffers and
    replays the captured graph (captured on the first call), returning the last hidden state
    [1, H] (a view of the step's buffer)."""

    def __init__(self, layers, H, NH, NKV, HD, lmax, theta=1e6, eps=1e-6, device=None, graph=True, pdl=True):
        self.layers = layers
        self.H, self.NH, self.NKV, self.HD, self.lmax, self.eps = H, NH, NKV, HD, lmax, float(eps)
        dev = layers[0].qkv.qweight.device if device is None else torch.device(device)
        self.dev = dev
        I = max(l.I for l in layers)
        self.h = torch.zeros((1, H), dtype=torch.float32, device=dev)
        self.qkv = torch.empty((1, (NH + 2 * NKV) * HD), dtype=torch.float32, device=dev)
        self.att = torch.empty((1, NH * HD), dtype=torch.float32, device=dev)
        self.gu = torch.empty((1, 2 * I), dtype=torch.float32, device=dev)
        self.pos = torch.zeros((1,), dtype=torch.int32, device=dev)
        self.kc = [torch.zeros((NKV, lmax, HD), dtype=torch.float32, device=dev) for _ in layers]
        self.vc = [torch.zeros((NKV, lmax, HD), dtype=torch.float32, device=dev) for _ in layers]
        c, s = rope_tables(lmax, HD, theta)
        self.cos = torch.from_numpy(c).to(dev)
        self.sin = torch.from_numpy(s).to(dev)
        self.scale = 1.0 / math.sqrt(HD)
        # attention partials and per-head counters (zero once; the kernel leaves them at zero)
        self.att_ws = torch.zeros(int(_ffi.fn("ql_decode_attention_workspace")(NH, HD, lmax)), dtype=torch.uint8,
                                  device=dev)
        self.use_graph = graph
        # programmatic dependent launch: each kernel of the step may start (and stream its weights)
        # while the previous one finishes; every kernel waits for the previous one's outputs
        self.pdl = bool(pdl)
        self.graph = None
        self.stream = None

    def launches_per_step(self):
        return 5 * len(self.layers)

    def _forward(self, stream=None):
        prev = _ffi.set_launch_flags(_ffi.LAUNCH_PDL if self.pdl else 0)
        try:
            return self._layers(stream)
        finally:
            _ffi.set_launch_flags(prev)

    def _layers(self, stream=None):
        h = self.h
        for i, lay in enumerate(self.layers):
            fused_linear(h, lay.qkv, norm_weight=lay.in_ln, norm_eps=self.eps, out=self.qkv, stream=stream)
            _ffi.call("ql_decode_attention", self.qkv.data_ptr(), self.NH, self.NKV, self.HD, self.cos.data_ptr(),
                      self.sin.data_ptr(), self.pos.data_ptr(), self.kc[i].data_ptr(), self.vc[i].data_ptr(),
                      self.lmax, self.scale, self.att.data_ptr(), self.att_ws.data_ptr(), self.att_ws.numel(),
                      _ffi.stream_ptr(stream, self.dev))
            fused_linear(self.att, lay.o, residual=h, out=h, stream=stream)
            fused_linear(h, lay.gate_up, norm_weight=lay.post_ln, norm_eps=self.eps, out=self.gu, stream=stream)
            gu = self.gu[:, :2 * lay.I]
            fused_linear(gu, lay.down, glu=lay.I, residual=h, out=h, stream=stream)
        return h

    def _capture(self):
        self.stream = torch.cuda.Stream(self.dev)
        self.stream.wait_stream(torch.cuda.current_stream(self.dev))
        h0 = self.h.clone()
        pos0 = self.pos.clone()
        kc0 = [k.clone() for k in self.kc]
        vc0 = [v.clone() for v in self.vc]
        with torch.cuda.stream(self.stream):
            self._forward(self.stream)          # warm-up (loads the kernels, sets attributes)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=self.stream):
                self._forward(self.stream)
        torch.cuda.current_stream(self.dev).wait_stream(self.stream)
        # the warm-up and capture ran the step: restore the state they changed
        self.h.copy_(h0)
        self.pos.copy_(pos0)
        for k, k0 in zip(self.kc, kc0):
            k.copy_(k0)
        for v, v0 in zip(self.vc, vc0):
            v.copy_(v0)

    def step(self, embedding, pos):
        """Run one token: embedding [H] (host or device), pos its position; returns h [1, H]."""
        if not 0 <= pos < self.lmax:
            raise ValueError("position %d outside the cache (lmax %d)" % (pos, self.lmax))
        e = torch.as_tensor(embedding, dtype=torch.float32).reshape(1, self.H)
        self.h.copy_(e.to(self.dev, non_blocking=True))
        self.pos.fill_(int(pos))
        if not self.use_graph:
            return self._forward()
        if self.graph is None:
            self._capture()
            self.h.copy_(e.to(self.dev, non_blocking=True))
            self.pos.fill_(int(pos))
        self.graph.replay()
        return self.h
