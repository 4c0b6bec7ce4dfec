"""On-disk formats either side of the quantized-linear path: AutoGPTQ safetensors checkpoints
and GGUF (llama.cpp) files. Tensors are read on the host (memory-mapped, one tensor at a time)
and handed to the GPU operators in their on-disk packing; nothing is dequantised on the way.

Reference counterparts (package `webtorch`):
  * safetensors header / tensor reads: llm.py:546-566 (`_hdr`, `_np`): 8-byte little-endian
    header length, JSON header {name: {dtype, shape, data_offsets}}, raw little-endian data;
    BF16 widened to fp32 by a 16-bit shift, F16 to fp32, I32 as is.
  * AutoGPTQ linear: llm.py:568-572 (`_qlin`) -> QuantizedLinear.from_autogptq. The reference
    never reads `g_idx` (a desc_act checkpoint would load with wrong groups); this loader passes
    it on, so act-order checkpoints run correctly.
  * AutoGPTQ writer: quantize.py:80-106 (`_quantize_raw`, `_pack_autogptq`) and the manifest of
    quantize.py:150 (quantization_config {bits, group_size, desc_act: False, sym: False}).
  * GGUF: ggufload.py:92-113 (`parse_header`), llm.py:731-783 (`_gexperts`, `_gload_native`):
    2-D weights uploaded unchanged, stacked experts [E, out, in] split per expert (blocks run
    along `in`, so every expert's slice is block-aligned).
"""
import json
import mmap
import os
import struct

import numpy as np
import torch

from . import _ffi

__all__ = ["SafeTensors", "SafeTensorsDir", "write_safetensors", "load_autogptq_linear", "autogptq_config",
           "quantize_autogptq", "write_autogptq", "GGUFFile", "GGML_TYPES", "gguf_tensor_nbytes",
           "gguf_linear", "gguf_experts"]

# ---------------------------------------------------------------------------------------
# safetensors
# ---------------------------------------------------------------------------------------
_ST_NP = {"F64": np.float64, "F32": np.float32, "F16": np.float16, "I64": np.int64, "I32": np.int32,
          "I16": np.int16, "I8": np.int8, "U8": np.uint8, "U16": np.uint16, "U32": np.uint32, "BOOL": np.bool_}
_NP_ST = {np.dtype(v): k for k, v in _ST_NP.items()}


class SafeTensors:
    """One safetensors file, memory-mapped. `numpy(name)` returns the tensor as stored (BF16 as
    fp32, the way the reference widens it); `raw(name)` the bytes."""

    def __init__(self, path):
        self.path = path
        self._fh = open(path, "rb")
        self._mm = mmap.mmap(self._fh.fileno(), 0, access=mmap.ACCESS_READ)
        n = struct.unpack("<Q", self._mm[:8])[0]
        if n > len(self._mm) - 8:
            raise ValueError("%s: safetensors header length %d exceeds the file" % (path, n))
        hdr = json.loads(bytes(self._mm[8:8 + n]).decode("utf-8"))
        self.metadata = hdr.pop("__metadata__", None) or {}
        self.header = hdr
        self.base = 8 + n

    def names(self):
        return list(self.header)

    def __contains__(self, name):
        return name in self.header

    def info(self, name):
        d = self.header[name]
        return d["dtype"], tuple(d["shape"])

    def raw(self, name):
        a, z = self.header[name]["data_offsets"]
        return memoryview(self._mm)[self.base + a:self.base + z]

    def numpy(self, name):
        dt, shape = self.info(name)
        raw = self.raw(name)
        if dt == "BF16":
            arr = (np.frombuffer(raw, np.uint16).astype(np.uint32) << 16).view(np.float32)
        elif dt in _ST_NP:
            arr = np.frombuffer(raw, _ST_NP[dt])
        else:
            raise NotImplementedError("safetensors dtype %s" % dt)
        return arr.reshape(shape)

    def close(self):
        """Release the mapping (left to the garbage collector while tensor views are alive)."""
        try:
            self._mm.close()
        except BufferError:
            pass
        self._fh.close()


class SafeTensorsDir:
    """A checkpoint directory: model.safetensors.index.json's weight_map over several shards, or a
    single model.safetensors (llm.py:629-633)."""

    def __init__(self, path):
        self.path = path
        idx = os.path.join(path, "model.safetensors.index.json")
        self._files = {}
        if os.path.exists(idx):
            with open(idx) as fh:
                self.weight_map = json.load(fh)["weight_map"]
        else:
            st = self._file("model.safetensors")
            self.weight_map = {k: "model.safetensors" for k in st.names()}

    def _file(self, fn):
        if fn not in self._files:
            self._files[fn] = SafeTensors(os.path.join(self.path, fn))
        return self._files[fn]

    def __contains__(self, name):
        return name in self.weight_map

    def numpy(self, name):
        return self._file(self.weight_map[name]).numpy(name)

    def config(self):
        with open(os.path.join(self.path, "config.json")) as fh:
            return json.load(fh)


def write_safetensors(path, tensors, metadata=None):
    """Write {name: array} (numpy or torch; bfloat16 torch tensors stay BF16) as safetensors."""
    hdr, blobs, off = {}, [], 0
    for name, t in tensors.items():
        if isinstance(t, torch.Tensor):
            t = t.detach().cpu().contiguous()
            if t.dtype == torch.bfloat16:
                b = t.view(torch.int16).numpy().tobytes()
                dt = "BF16"
            else:
                a = t.numpy()
                b, dt = a.tobytes(), _NP_ST[a.dtype]
            shape = list(t.shape)
        else:
            a = np.ascontiguousarray(t)
            b, dt, shape = a.tobytes(), _NP_ST[a.dtype], list(a.shape)
        hdr[name] = {"dtype": dt, "shape": shape, "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if metadata:
        hdr["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(hdr, separators=(",", ":")).encode("utf-8")
    h += b" " * ((-len(h)) % 8)
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(h)))
        fh.write(h)
        for b in blobs:
            fh.write(b)


# ---------------------------------------------------------------------------------------
# AutoGPTQ checkpoints
# ---------------------------------------------------------------------------------------
def autogptq_config(cfg):
    """(group_size, bits, desc_act) from a config.json dict's quantization_config."""
    q = cfg["quantization_config"]
    return int(q["group_size"]), int(q["bits"]), bool(q.get("desc_act", False))


def load_autogptq_linear(st, prefix, gs, bits, device=None):
    """The QuantizedLinear of `prefix` (.qweight / .qzeros / .scales, optional .bias and .g_idx)
    from a SafeTensors / SafeTensorsDir. A non-trivial g_idx (act-order checkpoint) is honoured:
    the rows are sorted by group once at load and x is gathered in the kernels."""
    from .qlinear import QuantizedLinear
    get = st.numpy
    b = get(prefix + ".bias") if (prefix + ".bias") in st else None
    g_idx = get(prefix + ".g_idx") if (prefix + ".g_idx") in st else None
    sc = get(prefix + ".scales")
    return QuantizedLinear.from_autogptq(get(prefix + ".qweight"), get(prefix + ".qzeros"), sc, b, gs, bits,
                                         g_idx=g_idx, device=device)


def quantize_autogptq(W_out_in, gs=128, bits=4, zero_store_offset=1, scales_dtype=torch.float16, device=None):
    """Quantise a dense (out, in) weight on the GPU into AutoGPTQ tensors (webtorch/quantize.py:
    80-106, bit-identical): returns dict(qweight [Kp/per, Np] int32, qzeros [Kp/gs, Np/per] int32
    storing zp - 1, scales [Kp/gs, Np] fp16, g_idx [Kp] int32 = k // gs) as torch tensors on the
    device. zero_store_offset=0 and scales_dtype=float32 give the reference's own packing
    (QuantizedLinear with zero_offset 0)."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if not isinstance(W_out_in, torch.Tensor):
        W_out_in = torch.from_numpy(np.ascontiguousarray(np.asarray(W_out_in)))
    W = W_out_in.to(dev)
    if W.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        W = W.float()
    W = W.contiguous()
    N, K = W.shape
    per = 32 // bits
    Kp = K + (-K) % gs
    Np = N + (-N) % per
    qw = torch.empty((Kp // per, Np), dtype=torch.int32, device=dev)
    qz = torch.empty((Kp // gs, Np // per), dtype=torch.int32, device=dev)
    sc = torch.empty((Kp // gs, Np), dtype=scales_dtype, device=dev)
    _ffi.call("ql_gptq_quantize", W.data_ptr(), _ffi.dtype_code(W.dtype), W.stride(0), N, K, gs, bits,
              int(zero_store_offset), qw.data_ptr(), qz.data_ptr(), sc.data_ptr(), _ffi.dtype_code(sc.dtype),
              _ffi.stream_ptr(None, dev))
    g_idx = torch.arange(Kp, dtype=torch.int32, device=dev) // gs
    return {"qweight": qw, "qzeros": qz, "scales": sc, "g_idx": g_idx, "K": K, "N": N, "Kp": Kp, "Np": Np}


def write_autogptq(path, weights, gs=128, bits=4, biases=None, device=None):
    """Quantise {prefix: (out, in) weight} on the GPU and write an AutoGPTQ safetensors file
    (<prefix>.qweight / .qzeros / .scales / .g_idx, and .bias as fp16 when given), the layout
    transformers / auto_gptq / vLLM load. Returns the quantization_config to put in config.json
    (quantize.py:150)."""
    out = {}
    for prefix, W in weights.items():
        p = quantize_autogptq(W, gs, bits, device=device)
        for k in ("qweight", "qzeros", "scales", "g_idx"):
            out[prefix + "." + k] = p[k]
        if biases and prefix in biases:
            b = biases[prefix]
            b = b if isinstance(b, torch.Tensor) else torch.from_numpy(np.asarray(b))
            out[prefix + ".bias"] = b.to(torch.float16)
    write_safetensors(path, out)
    return {"bits": bits, "group_size": gs, "desc_act": False, "sym": False, "quant_method": "gptq"}


# ---------------------------------------------------------------------------------------
# GGUF
# ---------------------------------------------------------------------------------------
GGUF_MAGIC = 0x46554747   # "GGUF" little-endian

# ggml tensor types: id -> (name, values per block, bytes per block)
GGML_TYPES = {0: ("F32", 1, 4), 1: ("F16", 1, 2), 2: ("Q4_0", 32, 18), 3: ("Q4_1", 32, 20), 6: ("Q5_0", 32, 22),
              7: ("Q5_1", 32, 24), 8: ("Q8_0", 32, 34), 9: ("Q8_1", 32, 36), 10: ("Q2_K", 256, 84),
              11: ("Q3_K", 256, 110), 12: ("Q4_K", 256, 144), 13: ("Q5_K", 256, 176), 14: ("Q6_K", 256, 210),
              15: ("Q8_K", 256, 292), 30: ("BF16", 1, 2)}
GGML_IDS = {v[0]: k for k, v in GGML_TYPES.items()}

# metadata value types
_GT_U8, _GT_I8, _GT_U16, _GT_I16, _GT_U32, _GT_I32, _GT_F32, _GT_BOOL, _GT_STR, _GT_ARR, _GT_U64, _GT_I64, \
    _GT_F64 = range(13)
_GT_FMT = {_GT_U8: "<B", _GT_I8: "<b", _GT_U16: "<H", _GT_I16: "<h", _GT_U32: "<I", _GT_I32: "<i", _GT_F32: "<f",
           _GT_BOOL: "<?", _GT_U64: "<Q", _GT_I64: "<q", _GT_F64: "<d"}


def gguf_tensor_nbytes(ttype, n):
    """Bytes of n values of ggml type `ttype` (n a whole number of blocks)."""
    if ttype not in GGML_TYPES:
        raise NotImplementedError("ggml type %d" % ttype)
    _, vals, nbytes = GGML_TYPES[ttype]
    if n % vals:
        raise ValueError("%d values are not whole %s blocks" % (n, GGML_TYPES[ttype][0]))
    return n // vals * nbytes


class GGUFFile:
    """A GGUF file, memory-mapped: version, metadata, tensor infos (dims in ggml order, innermost
    first), data_start; `raw(name)` returns a tensor's bytes."""

    def __init__(self, path):
        self.path = path
        self._fh = open(path, "rb")
        self._mm = mmap.mmap(self._fh.fileno(), 0, access=mmap.ACCESS_READ)
        self._p = 0
        if self._u32() != GGUF_MAGIC:
            raise ValueError("%s is not a GGUF file" % path)
        self.version = self._u32()
        n_tensors, n_kv = self._u64(), self._u64()
        self.metadata = {}
        for _ in range(n_kv):
            key = self._str()
            self.metadata[key] = self._value(self._u32())
        self.tensors = {}
        for _ in range(n_tensors):
            name = self._str()
            nd = self._u32()
            dims = [self._u64() for _ in range(nd)]
            ttype = self._u32()
            off = self._u64()
            self.tensors[name] = {"dims": dims, "type": ttype, "offset": off}
        align = int(self.metadata.get("general.alignment", 32))
        self.data_start = (self._p + align - 1) // align * align

    # --- header reads ---
    def _take(self, n):
        if self._p + n > len(self._mm):
            raise EOFError("GGUF header runs past the end of %s" % self.path)
        b = self._mm[self._p:self._p + n]
        self._p += n
        return b

    def _u32(self):
        return struct.unpack("<I", self._take(4))[0]

    def _u64(self):
        return struct.unpack("<Q", self._take(8))[0]

    def _str(self):
        return self._take(self._u64()).decode("utf-8", "replace")

    def _value(self, t):
        if t == _GT_STR:
            return self._str()
        if t == _GT_ARR:
            at, n = self._u32(), self._u64()
            return [self._value(at) for _ in range(n)]
        if t not in _GT_FMT:
            raise ValueError("bad GGUF metadata type %d" % t)
        fmt = _GT_FMT[t]
        return struct.unpack(fmt, self._take(struct.calcsize(fmt)))[0]

    # --- tensors ---
    def type_name(self, name):
        return GGML_TYPES.get(self.tensors[name]["type"], (str(self.tensors[name]["type"]),))[0]

    def shape(self, name):
        """numpy order (outermost first)."""
        return tuple(int(d) for d in reversed(self.tensors[name]["dims"]))

    def raw(self, name):
        t = self.tensors[name]
        n = 1
        for d in t["dims"]:
            n *= int(d)
        a = self.data_start + int(t["offset"])
        return memoryview(self._mm)[a:a + gguf_tensor_nbytes(t["type"], n)]

    def close(self):
        """Release the mapping (left to the garbage collector while tensor views are alive)."""
        try:
            self._mm.close()
        except BufferError:
            pass
        self._fh.close()


def gguf_linear(gg, name, bias=None, device=None):
    """A 2-D GGUF weight (out, in) as a GGMLLinear over its bytes, unchanged (llm.py:762-783)."""
    from .ggml import GGMLLinear
    shape = gg.shape(name)
    if len(shape) != 2:
        raise ValueError("%s is not a 2-D weight (shape %s)" % (name, shape))
    N, K = shape
    return GGMLLinear(bytes(gg.raw(name)), gg.type_name(name), K, N, bias=bias, device=device)


def gguf_experts(gg, name, device=None):
    """The experts of a stacked [E, out, in] GGUF tensor (`ffn_*_exps`) as one GGMLLinear each: the
    packed bytes are read once and split per expert; quantisation blocks run along `in` and
    out * in is whole blocks, so every expert's slice is block-aligned (llm.py:731-760)."""
    from .ggml import GGMLLinear
    E, N, K = gg.shape(name)
    t = gg.tensors[name]
    per = gguf_tensor_nbytes(t["type"], N * K)
    raw = gg.raw(name)
    tn = gg.type_name(name)
    return [GGMLLinear(bytes(raw[e * per:(e + 1) * per]), tn, K, N, device=device) for e in range(E)]
