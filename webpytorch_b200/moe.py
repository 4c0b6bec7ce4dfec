"""Sparse mixture-of-experts MLP on B200: the drop-in for webtorch's `lm_engine.moe_mlp`.

Reference (webtorch/lm_engine.py:294-329): router logits -> float64 softmax over all experts ->
top-k (argpartition) -> optional renormalisation -> for every expert with routed tokens
`down(silu(gate(x)) * up(x))`, weighted and scatter-added -> plus an optional shared expert,
optionally gated by sigmoid(shared_gate(x)). The reference routes on the host and launches one
QuantizedLinear per expert and projection.

Here one forward is a fixed sequence of launches with no host round trip (so it can be
captured in a CUDA graph):
  ql_moe_route            device softmax / top-k / histogram / scan / scatter
  ql_moe_grouped_matmul          x rows gathered per expert @ stacked [gate | up] -> [P, 2I]
  ql_moe_grouped_matmul_swiglu   silu(gate) * up formed while staging, @ stacked down -> [P, H]
  (shared expert: the same two launches over one fused gate|up pack and its down)
  ql_moe_combine          weighted sum of each token's k rows (+ gated shared output)
P = T * top_k sorted (token, expert) rows. The grouped GEMMs read each expert's row count on
the device: decode steps (few rows per expert) run the split-K GEMV over active experts only,
prefill steps the tcgen05 GEMM over a device-built tile table.
"""
import torch

from . import _ffi
from .qlinear import QuantizedLinear, _device

__all__ = ["MoEBlock", "StackedExperts", "moe_mlp"]

TILE_ROWS = 128   # rows per tile of the grouped tensor-core GEMM


def _as_quantized(lin, what):
    if not isinstance(lin, QuantizedLinear):
        raise TypeError("%s must be a QuantizedLinear (got %s)" % (what, type(lin).__name__))
    if lin.x_perm is not None:
        raise NotImplementedError("%s: act-order (g_idx) experts are not supported in a grouped block" % what)
    if lin.Kp != lin.Kt or lin.Np != lin.Nt:
        raise NotImplementedError("%s: padded (Kp != Kt or Np != Nt) experts are not supported" % what)
    if lin.bias is not None and bool(torch.any(lin.bias != 0)):
        raise NotImplementedError("%s: expert biases are not supported" % what)
    return lin


class StackedExperts:
    """E experts' GPTQ packs of one projection, stacked contiguously: qweight [E, K/per, N],
    qzeros [E, K/gs, N/per], scales [E, K/gs, N]. `parts` lists per expert the projections that
    are concatenated along N (gate | up)."""

    def __init__(self, experts, parts, device=None):
        dev = _device(device)
        first = _as_quantized(experts[0][parts[0]], "experts[0].%s" % parts[0])
        self.K, self.gs, self.bits, self.zoff = first.Kp, first.gs, first.bits, first.zero_offset
        self.E = len(experts)
        per = 32 // self.bits
        qws, qzs, scs = [], [], []
        ns = []
        for i, ex in enumerate(experts):
            cols_w, cols_z, cols_s = [], [], []
            for p in parts:
                lin = _as_quantized(ex[p], "experts[%d].%s" % (i, p))
                if (lin.Kp, lin.gs, lin.bits, lin.zero_offset) != (self.K, self.gs, self.bits, self.zoff):
                    raise ValueError("experts[%d].%s: K, group size, bits and zero offset must match" % (i, p))
                if lin.Np % per and len(parts) > 1:
                    raise ValueError("fused projections need N %% %d == 0" % per)
                cols_w.append(lin.qweight)
                cols_z.append(lin.qzeros)
                cols_s.append(lin.scales)
            qws.append(torch.cat(cols_w, 1))
            qzs.append(torch.cat(cols_z, 1))
            scs.append(torch.cat([s.to(cols_s[0].dtype) for s in cols_s], 1))
            ns.append(qws[-1].shape[1])
        if len(set(ns)) != 1:
            raise ValueError("every expert must have the same output width")
        self.N = ns[0]
        self.qweight = torch.stack(qws).to(dev).contiguous()
        self.qzeros = torch.stack(qzs).to(dev).contiguous()
        self.scales = torch.stack(scs).to(dev).contiguous()

    @classmethod
    def from_packed(cls, qweight, qzeros, scales, gs, bits, zero_offset=1.0):
        """Wrap already-stacked device tensors: qweight [E, K/per, N], qzeros [E, K/gs, N/per],
        scales [E, K/gs, N] (AutoGPTQ packing per expert)."""
        self = cls.__new__(cls)
        per = 32 // bits
        self.E, kp, self.N = (int(v) for v in qweight.shape)
        self.K, self.gs, self.bits, self.zoff = kp * per, int(gs), int(bits), float(zero_offset)
        if tuple(qzeros.shape) != (self.E, self.K // gs, self.N // per) or \
                tuple(scales.shape) != (self.E, self.K // gs, self.N):
            raise ValueError("qzeros/scales shapes do not match qweight")
        self.qweight, self.qzeros, self.scales = qweight.contiguous(), qzeros.contiguous(), scales.contiguous()
        return self

    def nbytes(self):
        return int(self.qweight.numel() * 4 + self.qzeros.numel() * 4 +
                   self.scales.numel() * self.scales.element_size())

    def expert_nbytes(self):
        return self.nbytes() // self.E


def tile_rows_for(P, E, K, gs, max_rows):
    """Tile height of the routing table the grouped matmul wants for this call (32 / 64 / 128 for
    the tensor-core GEMM, 4 or 8 for the decode GEMV)."""
    return _ffi.load().ql_moe_tile_rows(P, E, K, gs, max_rows)


class Routing:
    """Device buffers written by ql_moe_route for T tokens."""

    def __init__(self, T, E, top_k, device, tile_rows=TILE_ROWS):
        P = T * top_k
        i32 = dict(dtype=torch.int32, device=device)
        self.T, self.E, self.top_k, self.P = T, E, top_k, P
        self.tile_rows = tile_rows
        self.topk_idx = torch.empty((T, top_k), **i32)
        self.topk_w = torch.empty((T, top_k), dtype=torch.float32, device=device)
        self.counts = torch.empty(E, **i32)
        self.offsets = torch.empty(E + 1, **i32)
        self.cursor = torch.empty(E, **i32)
        self.active = torch.empty(E, **i32)
        self.n_active = torch.empty(1, **i32)
        self.max_tiles = P // tile_rows + min(E, P) + 1
        self.tiles = torch.empty(2 * self.max_tiles, **i32)
        self.n_tiles = torch.empty(1, **i32)
        self.row_token = torch.empty(max(P, 1), **i32)
        self.pair_row = torch.empty((T, top_k), **i32)


def route(logits, top_k, norm_topk_prob=True, tile_rows=TILE_ROWS, stream=None):
    """Device routing of [T, E] fp32 logits (lm_engine.py:299-307); returns a Routing whose tile
    table has tiles of `tile_rows` rows."""
    if logits.dim() != 2:
        raise ValueError("logits must be [T, E]")
    logits = logits.to(torch.float32).contiguous()
    T, E = logits.shape
    r = Routing(T, E, top_k, logits.device, tile_rows)
    _ffi.call("ql_moe_route", _ffi.ptr(logits), T, E, top_k, int(bool(norm_topk_prob)), tile_rows,
              _ffi.ptr(r.topk_idx), _ffi.ptr(r.topk_w), _ffi.ptr(r.counts), _ffi.ptr(r.offsets),
              _ffi.ptr(r.cursor), _ffi.ptr(r.active), _ffi.ptr(r.n_active), _ffi.ptr(r.tiles),
              _ffi.ptr(r.n_tiles), r.max_tiles, _ffi.ptr(r.row_token), _ffi.ptr(r.pair_row),
              _ffi.stream_ptr(stream))
    return r


def grouped_matmul(x, row_token, r, w, out_dtype=torch.float32, stream=None):
    """y[P, N]: sorted row p of expert e = x[row_token[p]] (or x[p] when row_token is None) @ W_e."""
    if x.stride(-1) != 1:
        x = x.contiguous()
    P = r.P
    y = torch.empty((P, w.N), dtype=out_dtype, device=x.device)
    lib = _ffi.load()
    ws_bytes = lib.ql_moe_grouped_workspace(P, w.E, w.K, w.gs)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device) if ws_bytes else None
    _ffi.call("ql_moe_grouped_matmul", _ffi.ptr(x), _ffi.dtype_code(x.dtype), x.stride(0), _ffi.ptr(row_token),
              P, _ffi.ptr(w.qweight), _ffi.ptr(w.qzeros), _ffi.ptr(w.scales), _ffi.dtype_code(w.scales.dtype),
              w.E, _ffi.ptr(r.offsets), _ffi.ptr(r.active), _ffi.ptr(r.n_active), _ffi.ptr(r.tiles),
              _ffi.ptr(r.n_tiles), r.max_tiles, r.tile_rows, r.T, _ffi.ptr(y), _ffi.dtype_code(y.dtype),
              y.stride(0), w.K, w.N, w.gs, w.bits, float(w.zoff), _ffi.ptr(ws), ws_bytes, _ffi.stream_ptr(stream))
    return y


def down_swiglu(y, r, w, out_dtype=torch.float32, stream=None):
    """z[P, N] = (silu(y[:, :K]) * y[:, K:]) @ W_e per expert segment, the activation formed while
    staging (no [P, K] intermediate): per CTA in the decode GEMV, in the fp16 staging pass of the
    tensor-core GEMM."""
    P = r.P
    z = torch.empty((P, w.N), dtype=out_dtype, device=y.device)
    ws_bytes = _ffi.load().ql_moe_grouped_workspace(P, w.E, w.K, w.gs)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=y.device) if ws_bytes else None
    _ffi.call("ql_moe_grouped_matmul_swiglu", _ffi.ptr(y), _ffi.dtype_code(y.dtype), y.stride(0), P,
              _ffi.ptr(w.qweight), _ffi.ptr(w.qzeros), _ffi.ptr(w.scales), _ffi.dtype_code(w.scales.dtype), w.E,
              _ffi.ptr(r.offsets), _ffi.ptr(r.active), _ffi.ptr(r.n_active), _ffi.ptr(r.tiles), _ffi.ptr(r.n_tiles),
              r.max_tiles, r.tile_rows, r.T, _ffi.ptr(z), _ffi.dtype_code(z.dtype), z.stride(0), w.K, w.N, w.gs,
              w.bits, float(w.zoff), _ffi.ptr(ws), ws_bytes, _ffi.stream_ptr(stream))
    return z


def act(y, I, out_dtype=torch.float32, stream=None):
    """a[P, I] = silu(y[:, :I]) * y[:, I:] for the fused gate|up output y [P, 2I] (fp32)."""
    P = y.shape[0]
    a = torch.empty((P, I), dtype=out_dtype, device=y.device)
    _ffi.call("ql_moe_act", _ffi.ptr(y), P, I, _ffi.ptr(a), _ffi.dtype_code(a.dtype), _ffi.stream_ptr(stream))
    return a


class MoEBlock(torch.nn.Module):
    """The reference's `lay['moe']` block: dict(gate, experts=[{gate, up, down}], top_k,
    norm_topk_prob, shared=(gate, up, down) | None, shared_gate=callable | None).

    `gate` (the router) and `shared_gate` are any callables mapping a [T, H] device tensor to
    [T, E] / [T, 1] logits (a QuantizedLinear, a torch module, a lambda). Experts (and the
    shared expert) are QuantizedLinear layers with identical K, group size, bits and zero
    offset; they are restacked once at construction."""

    def __init__(self, gate, experts, top_k, norm_topk_prob=True, shared=None, shared_gate=None, device=None):
        super().__init__()
        dev = _device(device)
        self.router = gate
        self.top_k = int(top_k)
        self.norm_topk_prob = bool(norm_topk_prob)
        self.E = len(experts)
        if not 1 <= self.top_k <= min(self.E, 16):
            raise ValueError("top_k must be in 1..min(E, 16)")
        experts = [self._parts(e) for e in experts]
        self.gate_up = StackedExperts(experts, ("gate", "up"), dev)
        self.down = StackedExperts(experts, ("down",), dev)
        self.H = self.gate_up.K
        self.I = self.gate_up.N // 2
        if self.down.K != self.I or self.down.N != self.H:
            raise ValueError("down projections must map I=%d -> H=%d" % (self.I, self.H))
        self.shared = None
        self.shared_gate = shared_gate
        if shared:
            sp = self._parts(shared)
            self.shared = (StackedExperts([sp], ("gate", "up"), dev), StackedExperts([sp], ("down",), dev))
            self.SI = self.shared[0].N // 2

    @classmethod
    def from_stacked(cls, gate, gate_up, down, top_k, norm_topk_prob=True):
        """A block over pre-stacked StackedExperts (gate_up: [E] x [H -> 2I], down: [E] x [I -> H])."""
        self = cls.__new__(cls)
        torch.nn.Module.__init__(self)
        self.router, self.top_k, self.norm_topk_prob = gate, int(top_k), bool(norm_topk_prob)
        self.gate_up, self.down = gate_up, down
        self.E, self.H, self.I = gate_up.E, gate_up.K, gate_up.N // 2
        self.shared = self.shared_gate = None
        return self

    @staticmethod
    def _parts(e):
        if isinstance(e, dict):
            return {k: e[k] for k in ("gate", "up", "down")}
        g, u, d = e
        return {"gate": g, "up": u, "down": d}

    @staticmethod
    def from_layer(moe, device=None):
        """Build from the reference's layer dict (`lay['moe']`, lm_engine.py:296-298)."""
        return MoEBlock(moe["gate"], moe["experts"], moe["top_k"], moe.get("norm_topk_prob", True),
                        moe.get("shared"), moe.get("shared_gate"), device)

    def expert_ffn(self, x, r, stream=None):
        """Routed experts' outputs for the sorted rows: z [P, H] fp32."""
        y = grouped_matmul(x, r.row_token, r, self.gate_up, stream=stream)
        return down_swiglu(y, r, self.down, stream=stream)   # SwiGLU formed while staging

    def shared_ffn(self, x, stream=None):
        gu, dn = self.shared
        T = x.shape[0]
        r1 = _single_expert_routing(T, x.device, tile_rows_for(T, 1, gu.K, gu.gs, T))
        y = grouped_matmul(x, None, r1, gu, stream=stream)
        return down_swiglu(y, r1, dn, stream=stream)

    def forward(self, x, out_dtype=torch.float32, stream=None):
        """x [T, H] (fp32/fp16/bf16 on the GPU) -> [T, H] in out_dtype (fp32 as the reference)."""
        if x.dim() != 2 or x.shape[1] != self.H:
            raise ValueError("x must be [T, %d]" % self.H)
        T = x.shape[0]
        logits = self.router(x)
        logits = torch.as_tensor(logits, device=x.device).reshape(T, self.E)
        tr = tile_rows_for(T * self.top_k, self.E, self.H, self.gate_up.gs, T)
        r = route(logits, self.top_k, self.norm_topk_prob, tr, stream)
        z = self.expert_ffn(x, r, stream)
        ys = g = None
        if self.shared is not None:
            ys = self.shared_ffn(x, stream)
            if self.shared_gate is not None:
                g = torch.as_tensor(self.shared_gate(x), device=x.device).to(torch.float32).reshape(T, 1)
                g = g.contiguous()
        out = torch.empty((T, self.H), dtype=out_dtype, device=x.device)
        _ffi.call("ql_moe_combine", _ffi.ptr(z), _ffi.ptr(r.pair_row), _ffi.ptr(r.topk_w), T, self.top_k, self.H,
                  _ffi.ptr(ys), ys.stride(0) if ys is not None else 0, _ffi.ptr(g), 1 if g is not None else 0,
                  _ffi.ptr(out), _ffi.dtype_code(out.dtype), out.stride(0), _ffi.stream_ptr(stream))
        return out

    def nbytes(self):
        n = self.gate_up.nbytes() + self.down.nbytes()
        if self.shared is not None:
            n += self.shared[0].nbytes() + self.shared[1].nbytes()
        return n


_single_cache = {}


def _single_expert_routing(T, device, tile_rows=TILE_ROWS):
    """Routing of T tokens to one expert in token order (the shared expert): static buffers."""
    key = (T, str(device), tile_rows)
    r = _single_cache.get(key)
    if r is None:
        r = Routing(T, 1, 1, device, tile_rows)
        r.offsets.copy_(torch.tensor([0, T], dtype=torch.int32))
        r.active.zero_()
        r.n_active.fill_(1 if T else 0)
        n = (T + tile_rows - 1) // tile_rows
        tiles = torch.zeros(2 * r.max_tiles, dtype=torch.int32)
        tiles[0:2 * n:2] = 0
        tiles[1:2 * n:2] = torch.arange(n, dtype=torch.int32) * tile_rows
        r.tiles.copy_(tiles)
        r.n_tiles.fill_(n)
        _single_cache[key] = r
    return r


def moe_mlp(lm, lay, x):
    """Function-level drop-in for lm_engine.moe_mlp(lm, lay, x) (lm_engine.py:294): builds (and
    caches on the layer dict) the stacked block, then runs it."""
    blk = lay.get("_b200_block")
    if blk is None:
        blk = MoEBlock.from_layer(lay["moe"], device=x.device if isinstance(x, torch.Tensor) else None)
        lay["_b200_block"] = blk
    return blk(x)
