"""GPTQ quantized linear: the drop-in for webtorch's `QuantizedLinear` / `_gptq_matmul`.

Interface parity with the reference (webtorch/_core.py:4409-4459):
  * `QuantizedLinear(qweight, qzeros, scales, bias, Kt, Nt, Kp, Np, gs, bits, zero_offset=0.0)`
  * `QuantizedLinear.from_autogptq(qweight, qzeros, scales, bias, gs, bits)` sets
    zero_offset=1.0 (AutoGPTQ stores zero-1); an optional `g_idx` adds desc_act support,
    which the reference lacks (it hard-codes g = k // gs, _core.py:4056).
  * `QuantizedLinear.from_linear(lin, group_size=32, bits=4)`.
  * `ql(x)` -> `forward(x: [..., Kt]) -> [..., Nt]` in fp32 (the reference's output dtype), with
    Kp/Np padding and bias handled as in _core.py:4446-4456.
  * `_gptq_matmul(xf, qweight, qzeros, scales, K, N, gs, bits, zoff)` is the function-level
    boundary of _core.py:4008.

Weights live on the GPU as torch tensors in the AutoGPTQ packing, unchanged. Every product
runs in libqlinear.so (sm_100a); there is no CPU path.
"""
import numpy as np
import torch

from . import _ffi

__all__ = ["QuantizedLinear", "gptq_dequant", "_gptq_matmul", "gptq_quantize"]


def _device(device=None):
    if device is not None:
        return torch.device(device)
    if not torch.cuda.is_available():
        raise RuntimeError("webpytorch_b200 needs a CUDA device (B200, sm_100a); none is visible")
    return torch.device("cuda", torch.cuda.current_device())


def _to_dev(a, dtype, device):
    if isinstance(a, torch.Tensor):
        return a.to(device=device, dtype=dtype).contiguous()
    a = np.ascontiguousarray(np.asarray(a))
    if not a.flags.writeable:     # e.g. a view of a memory-mapped checkpoint
        a = a.copy()
    return torch.from_numpy(a).to(device=device, dtype=dtype).contiguous()


def _param_array(p):
    """The array behind a parameter: a torch tensor, a numpy array, or an object with `.data`
    holding one (the reference's Parameter). numpy's own `.data` is a raw buffer, not this."""
    if isinstance(p, (torch.Tensor, np.ndarray)):
        return p.detach() if isinstance(p, torch.Tensor) else p
    d = getattr(p, "data", p)
    return d.detach() if isinstance(d, torch.Tensor) else np.asarray(d)


def _scale_tensor(scales, device):
    """Scales keep their on-disk precision (fp16 for AutoGPTQ, fp32 for the reference quantizer)."""
    if isinstance(scales, torch.Tensor):
        dt = scales.dtype if scales.dtype in (torch.float16, torch.bfloat16, torch.float32) else torch.float32
        return scales.to(device=device, dtype=dt).contiguous()
    a = np.asarray(scales)
    if not a.flags.writeable:
        a = a.copy()
    dt = torch.float16 if a.dtype == np.float16 else torch.float32
    return torch.from_numpy(np.ascontiguousarray(a.astype(np.float16 if dt == torch.float16 else np.float32))
                            ).to(device).contiguous()


def gptq_dequant(qweight, qzeros, scales, K, N, gs, bits, zoff=0.0, g_idx=None, stream=None):
    """Exact fp32 [K, N] dequantisation on the GPU (bit-identical to the reference's unpack)."""
    W = torch.empty((K, N), dtype=torch.float32, device=qweight.device)
    _ffi.call("ql_gptq_dequant", _ffi.ptr(qweight), _ffi.ptr(qzeros), _ffi.ptr(scales),
              _ffi.dtype_code(scales.dtype), _ffi.ptr(g_idx), _ffi.ptr(W), K, N, gs, bits,
              float(zoff), _ffi.stream_ptr(stream))
    return W


_ws_cache = {}


def _workspace_bytes(M, K):
    """ql_gptq_matmul_workspace(M, K), remembered per shape."""
    n = _ws_cache.get((M, K))
    if n is None:
        n = _ws_cache[(M, K)] = int(_ffi.fn("ql_gptq_matmul_workspace")(M, K))
    return n


def _gptq_matmul(xf, qweight, qzeros, scales, K, N, gs, bits, zoff=0.0, *, x_perm=None, bias=None,
                 out=None, out_dtype=torch.float32, stream=None):
    """y[M, N] = xf[M, K] @ dequant(qweight, qzeros, scales) (+ bias), on the GPU.

    Mirrors webtorch/_core.py:4008 (`_gptq_matmul`); `xf` may be fp32, fp16 or bf16 and is
    read with its row stride (it must be contiguous along K)."""
    if xf.dim() != 2 or xf.shape[1] != K:
        raise ValueError("x must be [M, %d], got %s" % (K, tuple(xf.shape)))
    if xf.stride(1) != 1:
        xf = xf.contiguous()
    M = xf.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=xf.device)
    # calls of more than 4 tokens stage x in a workspace (the tensor-core path's fp16 copy or the
    # decode path's MMA operand); take it from torch's allocator
    ws_bytes = _workspace_bytes(M, K) if M > 4 else 0
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=xf.device) if ws_bytes else None
    _ffi.call("ql_gptq_matmul_ws", xf.data_ptr(), _ffi.dtype_code(xf.dtype), xf.stride(0), _ffi.ptr(x_perm),
              qweight.data_ptr(), qzeros.data_ptr(), scales.data_ptr(), _ffi.dtype_code(scales.dtype),
              _ffi.ptr(bias), out.data_ptr(), _ffi.dtype_code(out.dtype), out.stride(0), M, K, N, gs, bits,
              float(zoff), _ffi.ptr(ws), ws_bytes, _ffi.stream_ptr(stream, xf.device))
    return out


def gptq_quantize(W, group_size=32, bits=4):
    """Asymmetric min/max group quantiser on the GPU, restating webtorch/_core.py:3782-3824.

    W is [K, N] (in, out). Returns (qweight int32 [K/per, N], qzeros int32 [K/gs, N/per],
    scales fp32 [K/gs, N], K, N) in the reference's own packing (zero offset 0). Arithmetic
    runs in W's dtype (float64 stays float64, as the reference's numpy code does)."""
    if W.dtype != torch.float64:
        W = W.to(torch.float32)
    K, N = W.shape
    per = 32 // bits
    qmax = (1 << bits) - 1
    if K % group_size or K % per or N % per:
        raise ValueError("dims must divide group/pack size")
    nG = K // group_size
    blk = W.reshape(nG, group_size, N)
    wmin = blk.amin(1)
    wmax = blk.amax(1)
    # divide by a tensor: torch turns division by a Python scalar into a reciprocal multiply,
    # which is not the correctly rounded quotient numpy computes
    sc = (wmax - wmin) / torch.full_like(wmax, float(qmax))
    sc = torch.where(sc == 0, torch.full_like(sc, 1e-8), sc)
    zp = torch.clamp(torch.round(-wmin / sc), 0, qmax).to(torch.int32)
    q = torch.clamp(torch.round(blk / sc[:, None, :]) + zp[:, None, :], 0, qmax).to(torch.int64)
    q = q.reshape(K // per, per, N)
    sh = (torch.arange(per, device=W.device, dtype=torch.int64) * bits).view(1, per, 1)
    qweight = torch.sum(q << sh, dim=1, dtype=torch.int64)
    qweight = torch.where(qweight >= 2 ** 31, qweight - 2 ** 32, qweight).to(torch.int32)
    zs = zp.to(torch.int64).reshape(nG, N // per, per) << sh.view(1, 1, per)
    qzeros = torch.sum(zs, dim=2, dtype=torch.int64)
    qzeros = torch.where(qzeros >= 2 ** 31, qzeros - 2 ** 32, qzeros).to(torch.int32)
    return qweight.contiguous(), qzeros.contiguous(), sc.to(torch.float32).contiguous(), K, N


class QuantizedLinear(torch.nn.Module):
    """Inference-only GPTQ-format weight-quantized linear (group-wise int4/int8) on B200."""

    def __init__(self, qweight, qzeros, scales, bias, Kt, Nt, Kp, Np, gs, bits, zero_offset=0.0,
                 g_idx=None, device=None):
        super().__init__()
        dev = _device(device)
        self.Kt, self.Nt, self.Kp, self.Np = int(Kt), int(Nt), int(Kp), int(Np)
        self.gs, self.bits = int(gs), int(bits)
        self.zero_offset = float(zero_offset)   # AutoGPTQ stores (zero-1) -> use 1.0
        per = 32 // self.bits
        qw = _to_dev(qweight, torch.int32, dev)
        qz = _to_dev(qzeros, torch.int32, dev)
        sc = _scale_tensor(scales, dev)
        if tuple(qw.shape) != (self.Kp // per, self.Np):
            raise ValueError("qweight shape %s != (%d, %d)" % (tuple(qw.shape), self.Kp // per, self.Np))
        x_perm = None
        if g_idx is not None:
            x_perm, qw = self._desc_act(qw, g_idx, dev)
        self.register_buffer("qweight", qw)
        self.register_buffer("qzeros", qz)
        self.register_buffer("scales", sc)
        self.register_buffer("x_perm", x_perm)
        b = None
        if bias is not None:
            b = _to_dev(bias, torch.float32, dev)
            if b.numel() != self.Nt:
                raise ValueError("bias must have %d elements" % self.Nt)
            if self.Np != self.Nt:
                b = torch.cat([b, torch.zeros(self.Np - self.Nt, device=dev)])
        self.register_buffer("bias", b)

    def _desc_act(self, qw, g_idx, dev):
        """Sort rows so every group is a contiguous run; remember the x gather that undoes it."""
        gi = _to_dev(g_idx, torch.int64, dev)
        if gi.numel() != self.Kp:
            raise ValueError("g_idx must have Kp=%d entries" % self.Kp)
        trivial = torch.arange(self.Kp, device=dev) // self.gs
        if torch.equal(gi, trivial):
            return None, qw
        perm = torch.sort(gi, stable=True).indices
        if not torch.equal(gi[perm], trivial):
            raise NotImplementedError("g_idx whose groups are not all of size gs is not supported")
        perm32 = perm.to(torch.int32).contiguous()
        out = torch.empty_like(qw)
        _ffi.call("ql_gptq_sort_rows", _ffi.ptr(qw), _ffi.ptr(perm32), _ffi.ptr(out), self.Kp, self.Np,
                  self.bits, _ffi.stream_ptr())
        return perm32, out

    @staticmethod
    def from_autogptq(qweight, qzeros, scales, bias, gs, bits, g_idx=None, device=None):
        """Load AutoGPTQ int4/int8 tensors directly: qweight (K/per, N) int32, qzeros
        (K/gs, N/per) int32, scales (K/gs, N), bias (N,) or None, optional g_idx (K,)."""
        per = 32 // bits
        K = int(qweight.shape[0]) * per
        N = int(qweight.shape[1])
        return QuantizedLinear(qweight, qzeros, scales, bias, K, N, K, N, gs, bits, zero_offset=1.0,
                               g_idx=g_idx, device=device)

    @staticmethod
    def from_linear(lin, group_size=32, bits=4, device=None):
        """Quantise a linear layer whose `weight` is (K, N) = (in, out), as the reference's
        `Linear` stores it (webtorch/_core.py:472-477, 4432-4444)."""
        dev = _device(device)
        W = _param_array(lin.weight)
        wdt = torch.float64 if W.dtype in (torch.float64, np.float64) else torch.float32
        W = _to_dev(W, wdt, dev)
        b = getattr(lin, "bias", None)
        if b is not None:
            b = _param_array(b)
        K, N = W.shape
        per = 32 // bits
        kmul = group_size if group_size % per == 0 else group_size * per
        Kp = K + (-K) % kmul
        Np = N + (-N) % per
        if Kp != K or Np != N:
            W = torch.nn.functional.pad(W, (0, Np - N, 0, Kp - K))
        qw, qz, sc, _, _ = gptq_quantize(W, group_size, bits)
        if b is None:
            b = torch.zeros(N)
        return QuantizedLinear(qw, qz, sc, b, K, N, Kp, Np, group_size, bits, device=dev)

    def dequantized(self):
        """Exact fp32 [Kp, Np] weight (in the stored row order)."""
        return gptq_dequant(self.qweight, self.qzeros, self.scales, self.Kp, self.Np, self.gs, self.bits,
                            self.zero_offset)

    def forward(self, x, out_dtype=torch.float32, out=None):
        """y = x @ W + b for x [..., Kt] (fp32/fp16/bf16, on the GPU or the host)."""
        host = not x.is_cuda
        xd = x.to(self.qweight.device, non_blocking=True) if host else x
        lead = xd.shape[:-1]
        xf = xd.reshape(-1, self.Kt)
        if self.Kp != self.Kt:
            xf = torch.nn.functional.pad(xf, (0, self.Kp - self.Kt))
        M = xf.shape[0]
        direct = out is not None and self.Np == self.Nt and not host
        y = out.view(M, self.Nt) if direct else None
        y = _gptq_matmul(xf, self.qweight, self.qzeros, self.scales, self.Kp, self.Np, self.gs, self.bits,
                         self.zero_offset, x_perm=self.x_perm, bias=self.bias, out=y, out_dtype=out_dtype)
        if self.Np != self.Nt:
            y = y[:, :self.Nt].contiguous()
        y = y.reshape(*lead, self.Nt)
        if host:
            y = y.cpu()
        if out is not None and not direct:
            out.copy_(y.reshape(out.shape))
            return out
        return y

    def nbytes(self):
        n = self.qweight.numel() * 4 + self.qzeros.numel() * 4 + self.scales.numel() * self.scales.element_size()
        if self.bias is not None:
            n += self.bias.numel() * 4
        return int(n)
