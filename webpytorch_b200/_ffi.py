"""ctypes binding of libqlinear.so (the C ABI declared in include/qlinear.h).

There is no fallback: if the library is missing or a call fails, this raises.
"""
import ctypes
import os

from . import _build

F32, F16, BF16 = 0, 1, 2
_STATUS = {0: "ok", 1: "bad argument", 2: "misaligned", 3: "unsupported", 4: "CUDA error",
           5: "device wait timed out"}

_lib = None

_c_int, _c_long, _c_float = ctypes.c_int, ctypes.c_long, ctypes.c_float
_vp = ctypes.c_void_p

# name -> (restype, argtypes); mirrors include/qlinear.h
SIGNATURES = {
    "ql_version": (_c_int, []),
    "ql_last_error": (ctypes.c_char_p, []),
    "ql_gptq_dequant": (_c_int, [_vp, _vp, _vp, _c_int, _vp, _vp, _c_int, _c_int, _c_int, _c_int,
                                 _c_float, _vp]),
    "ql_gptq_matmul": (_c_int, [_vp, _c_int, _c_long, _vp, _vp, _vp, _vp, _c_int, _vp, _vp, _c_int,
                                _c_long, _c_int, _c_int, _c_int, _c_int, _c_int, _c_float, _vp]),
    "ql_gptq_sort_rows": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_int, _vp]),
    "ql_set_launch_flags": (_c_int, [_c_int]),
    "ql_gptq_matmul_workspace": (ctypes.c_size_t, [_c_int, _c_int]),
    "ql_gptq_matmul_ws": (_c_int, [_vp, _c_int, _c_long, _vp, _vp, _vp, _vp, _c_int, _vp, _vp, _c_int,
                                   _c_long, _c_int, _c_int, _c_int, _c_int, _c_int, _c_float, _vp,
                                   ctypes.c_size_t, _vp]),
    "ql_device_status": (_c_int, []),
    "ql_gptq_matmul_noalloc": (_c_int, [_vp, _c_int, _c_long, _vp, _vp, _vp, _vp, _c_int, _vp, _vp, _c_int,
                                        _c_long, _c_int, _c_int, _c_int, _c_int, _c_int, _c_float, _vp]),
    "ql_gptq_matmul_noalloc_max_scratch": (ctypes.c_size_t, []),
    "ql_q4k_dequant": (_c_int, [_vp, _vp, _c_int, _c_int, _vp]),
    "ql_q4k_matmul": (_c_int, [_vp, _c_int, _c_long, _vp, _vp, _vp, _c_int, _c_long, _c_int, _c_int, _c_int, _vp]),
    "ql_q4k_matmul_workspace": (ctypes.c_size_t, [_c_int, _c_int]),
    "ql_ggml_dequant": (_c_int, [_c_int, _vp, _vp, _c_int, _c_int, _vp]),
    "ql_ggml_matmul": (_c_int, [_vp, _c_int, _c_long, _vp, _c_int, _vp, _vp, _c_int, _c_long, _c_int, _c_int, _c_int,
                                _vp]),
    "ql_gptq_matmul_fused": (_c_int, [_vp, _c_int, _c_long, _vp, _vp, _vp, _vp, _c_int, _vp, _vp, _c_float, _c_int, _vp,
                                      _c_long, _vp, _c_int, _c_long, _c_int, _c_int, _c_int, _c_int, _c_int, _c_float,
                                      _vp, ctypes.c_size_t, _vp]),
    "ql_decode_attention": (_c_int, [_vp, _c_int, _c_int, _c_int, _vp, _vp, _vp, _vp, _vp, _c_int, _c_float, _vp, _vp,
                                     ctypes.c_size_t, _vp]),
    "ql_decode_attention_workspace": (ctypes.c_size_t, [_c_int, _c_int, _c_int]),
    "ql_gptq_quantize": (_c_int, [_vp, _c_int, _c_long, _c_int, _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp, _c_int,
                                  _vp]),
    "ql_q4k_matmul_ws": (_c_int, [_vp, _c_int, _c_long, _vp, _vp, _vp, _c_int, _c_long, _c_int, _c_int, _c_int, _vp,
                                  ctypes.c_size_t, _vp]),
    "ql_moe_route": (_c_int, [_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                              _vp, _vp, _c_int, _vp, _vp, _vp]),
    "ql_moe_group": (_c_int, [_vp, _c_int, _c_int, _c_int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_int, _vp, _vp,
                              _vp]),
    "ql_moe_grouped_workspace": (ctypes.c_size_t, [_c_long, _c_int, _c_int, _c_int]),
    "ql_moe_tile_rows": (_c_int, [_c_long, _c_int, _c_int, _c_int, _c_int]),
    "ql_moe_grouped_matmul": (_c_int, [_vp, _c_int, _c_long, _vp, _c_long, _vp, _vp, _vp, _c_int, _c_int, _vp,
                                       _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _vp, _c_int, _c_long, _c_int,
                                       _c_int, _c_int, _c_int, _c_float, _vp, ctypes.c_size_t, _vp]),
    "ql_moe_grouped_matmul_swiglu": (_c_int, [_vp, _c_int, _c_long, _c_long, _vp, _vp, _vp, _c_int, _c_int, _vp,
                                              _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _vp, _c_int, _c_long,
                                              _c_int, _c_int, _c_int, _c_int, _c_float, _vp, ctypes.c_size_t,
                                              _vp]),
    "ql_moe_act": (_c_int, [_vp, _c_long, _c_int, _vp, _c_int, _vp]),
    "ql_moe_combine": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_int, _vp, _c_long, _vp, _c_long, _vp, _c_int,
                                _c_long, _vp]),
}

LAUNCH_PDL = 1


def set_launch_flags(flags):
    """Process-wide launch flags (LAUNCH_PDL); returns the previous value."""
    return load().ql_set_launch_flags(int(flags))


class QLError(RuntimeError):
    """A libqlinear call returned a non-zero status."""

    def __init__(self, fn, code, msg):
        super().__init__("%s failed (%s): %s" % (fn, _STATUS.get(code, code), msg))
        self.code = code


def lib_path():
    return _build.LIB


def load(build_if_missing=True):
    """Load libqlinear.so, building it first if it is absent and nvcc is available."""
    global _lib
    if _lib is not None:
        return _lib
    path = _build.LIB
    if not os.path.exists(path):
        if not build_if_missing:
            raise RuntimeError("libqlinear.so is not built (run webpytorch_b200._build.build())")
        _build.build()
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


_fns = {}


def fn(name):
    """The bound ctypes function `name` (looked up once)."""
    f = _fns.get(name)
    if f is None:
        f = _fns[name] = getattr(load(), name)
    return f


def call(name, *args):
    rc = (_fns.get(name) or fn(name))(*args)
    if rc != 0:
        msg = _lib.ql_last_error()
        raise QLError(name, rc, msg.decode(errors="replace") if msg else "")
    return rc


def dtype_code(t):
    import torch
    m = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}
    if t not in m:
        raise TypeError("unsupported dtype %s (float32, float16 or bfloat16)" % t)
    return m[t]


def ptr(t):
    """Device address of a torch tensor (an int, which ctypes passes as void*), or None for None."""
    return None if t is None else t.data_ptr()


_raw_stream = None


def stream_ptr(stream=None, device=None):
    """The CUDA stream to launch on: `stream`, else torch's current stream on `device` (an index
    or torch.device; the current device when None). Read through torch's raw-stream query when it
    has one (no Stream object per call)."""
    global _raw_stream
    if stream is not None:
        return stream.cuda_stream
    import torch
    if _raw_stream is None:
        _raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", False)
    idx = device.index if isinstance(device, torch.device) else device
    if idx is None:
        idx = torch.cuda.current_device()
    if _raw_stream:
        return _raw_stream(idx)
    return torch.cuda.current_stream(idx).cuda_stream
