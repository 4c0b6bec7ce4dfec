"""GGUF quantised linear: the drop-in for webtorch's `GGMLLinear` / `ggml_matmul`.

Interface parity with the reference (webtorch/_core.py:4377-4406, 3720-3734):
  * `GGMLLinear(raw, type_name, K, N, bias=None)` takes the tensor's bytes exactly as the GGUF
    file stores them ([N rows] x [K / block] blocks; Q4_K: 256 values in 144 bytes).
  * `forward(x: [..., K]) -> [..., N]` in fp32, plus bias.
  * `ggml_matmul(xf, raw, type_name, K, N)` is the function-level boundary.

The bytes go to the GPU unchanged (no transpose: the CUDA kernels read the file's row layout)
and are decoded inside the matmul. Native kernels: Q4_K (TMA-fed integer-MMA GEMV), Q8_0, Q5_K
and Q6_K (the types of Q4_K_M / Q5_K_M / Q8_0 files, webtorch/_core.py:3071-3177). Other ggml
types raise NotImplementedError.
"""
import numpy as np
import torch

from . import _ffi

__all__ = ["GGMLLinear", "ggml_matmul", "q4k_dequant", "ggml_dequant", "NATIVE_TYPES"]

# values per block, bytes per block, ggml type id
NATIVE_TYPES = {"Q4_K": (256, 144, 12), "Q8_0": (32, 34, 8), "Q5_K": (256, 176, 13), "Q6_K": (256, 210, 14)}


def _device(device=None):
    if device is not None:
        return torch.device(device)
    if not torch.cuda.is_available():
        raise RuntimeError("webpytorch_b200 needs a CUDA device (B200, sm_100a); none is visible")
    return torch.device("cuda", torch.cuda.current_device())


def q4k_dequant(raw, K, N, stream=None):
    """Exact fp32 [N, K] weight from raw Q4_K bytes on the GPU (bit-identical to ggufload.dequant)."""
    W = torch.empty((N, K), dtype=torch.float32, device=raw.device)
    _ffi.call("ql_q4k_dequant", _ffi.ptr(raw), _ffi.ptr(W), N, K, _ffi.stream_ptr(stream))
    return W


def ggml_dequant(raw, type_name, K, N, stream=None):
    """Exact fp32 [N, K] weight from raw GGUF bytes of a native type (bit-identical to
    ggufload.dequant)."""
    if type_name not in NATIVE_TYPES:
        raise NotImplementedError("no native B200 kernel for ggml type %s" % type_name)
    W = torch.empty((N, K), dtype=torch.float32, device=raw.device)
    _ffi.call("ql_ggml_dequant", NATIVE_TYPES[type_name][2], _ffi.ptr(raw), _ffi.ptr(W), N, K,
              _ffi.stream_ptr(stream))
    return W


def ggml_matmul(xf, raw, type_name, K, N, *, bias=None, out=None, out_dtype=torch.float32, stream=None):
    """y[M, N] = xf[M, K] @ W[N, K].T (+ bias) with W decoded from `raw` inside the kernel."""
    if type_name not in NATIVE_TYPES:
        raise NotImplementedError("no native B200 kernel for ggml type %s (native: %s)"
                                  % (type_name, sorted(NATIVE_TYPES)))
    if xf.dim() != 2 or xf.shape[1] != K:
        raise ValueError("x must be [M, %d], got %s" % (K, tuple(xf.shape)))
    if xf.stride(1) != 1:
        xf = xf.contiguous()
    M = xf.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=xf.device)
    if type_name == "Q4_K":
        _ffi.call("ql_q4k_matmul", _ffi.ptr(xf), _ffi.dtype_code(xf.dtype), xf.stride(0), _ffi.ptr(raw),
                  _ffi.ptr(bias), _ffi.ptr(out), _ffi.dtype_code(out.dtype), out.stride(0), M, K, N,
                  _ffi.stream_ptr(stream))
    else:
        _ffi.call("ql_ggml_matmul", _ffi.ptr(xf), _ffi.dtype_code(xf.dtype), xf.stride(0), _ffi.ptr(raw),
                  NATIVE_TYPES[type_name][2], _ffi.ptr(bias), _ffi.ptr(out), _ffi.dtype_code(out.dtype),
                  out.stride(0), M, K, N, _ffi.stream_ptr(stream))
    return out


class GGMLLinear(torch.nn.Module):
    """Inference-only linear whose weight stays in the encoding the GGUF file shipped it in."""

    def __init__(self, raw, type_name, K, N, bias=None, device=None):
        super().__init__()
        if type_name not in NATIVE_TYPES:
            raise NotImplementedError("no native B200 kernel for ggml type %s" % type_name)
        dev = _device(device)
        vals, blk, _ = NATIVE_TYPES[type_name]
        K, N = int(K), int(N)
        if K % vals:
            raise ValueError("K=%d is not a multiple of the %s block (%d)" % (K, type_name, vals))
        nbytes = N * (K // vals) * blk
        if isinstance(raw, torch.Tensor):
            b = raw.reshape(-1).to(torch.uint8)
        else:
            b = torch.from_numpy(np.frombuffer(bytes(raw) if not isinstance(raw, np.ndarray) else raw.tobytes(),
                                               np.uint8).copy())
        if b.numel() < nbytes:
            raise ValueError("raw holds %d bytes, %s [%d, %d] needs %d" % (b.numel(), type_name, N, K, nbytes))
        self.register_buffer("raw", b[:nbytes].to(dev).contiguous())
        self.type_name = type_name
        self.Kt, self.Nt = K, N
        self.register_buffer("bias", None if bias is None else
                             torch.as_tensor(np.asarray(bias, np.float32)).to(dev).contiguous())

    def dequantized(self):
        return ggml_dequant(self.raw, self.type_name, self.Kt, self.Nt)

    def forward(self, x, out_dtype=torch.float32, out=None):
        host = not x.is_cuda
        xd = x.to(self.raw.device, non_blocking=True) if host else x
        lead = xd.shape[:-1]
        xf = xd.reshape(-1, self.Kt)
        y = ggml_matmul(xf, self.raw, self.type_name, self.Kt, self.Nt, bias=self.bias,
                        out=None if out is None or host else out.view(-1, self.Nt), out_dtype=out_dtype)
        y = y.reshape(*lead, self.Nt)
        if host:
            y = y.cpu()
            if out is not None:
                out.copy_(y)
                return out
        return y
