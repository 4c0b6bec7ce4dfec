"""Multi-GPU forms of the quantized-linear path: one process per GPU, torch.distributed (NCCL).

* `ShardedQuantizedLinear` / `ShardedGGMLLinear`: the weight is split by output columns N
  (GPTQ: qweight[:, n0:n1], scales[:, n0:n1], qzeros[:, n0/per:n1/per]; Q4_K: rows n0:n1 of the
  GGUF tensor). x is replicated; each rank computes its slice with the single-GPU kernels and
  one all-gather assembles [M, N] on every rank. Shards are multiples of 32 columns (the GEMV
  strip width); the padded tail columns carry zero weights and are sliced away.
* `ExpertParallelMoE`: the experts are split across ranks (E / P each, expert e on rank
  e // (E / P)); every rank routes its own tokens, sends each (token, expert) pair's activation
  row to the expert's rank (counts all-to-all, then a variable all-to-all of the rows), runs its
  local experts as one grouped GEMM, sends the results back and combines them with the
  routing weights. The order of every exchange is fixed, so the result does not depend on the
  rank count beyond the expert FFN's own rounding.

The reference runs one device only (webtorch/_core.py:4008-4043 for the linear,
webtorch/lm_engine.py:294-329 for the MoE block); the partitioning follows its operators.

Compute goes through a backend object so that the collective choreography can be tested on CPU
with gloo: `CudaBackend` (the default) calls libqlinear; tests may pass their own.
"""
import torch
import torch.distributed as dist

from . import _ffi
from . import moe as _moe
from .qlinear import _gptq_matmul, _scale_tensor, _to_dev

__all__ = ["ShardedQuantizedLinear", "ShardedGGMLLinear", "ExpertParallelMoE", "CudaBackend", "shard_range"]

STRIP = 32   # GEMV column strip: shard widths are multiples of it


def _world(group):
    if not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def shard_range(N, P, r, align=STRIP):
    """Columns [n0, n1) of rank r when N is split P ways in multiples of `align` (equal widths
    w = ceil(N / P / align) * align; trailing ranks may hold fewer or no real columns)."""
    w = -(-N // P)
    w = -(-w // align) * align
    n0 = min(r * w, N)
    return n0, min(n0 + w, N), w


def _gather_columns(y_local, w, N, group):
    """[M, w] slices of all ranks -> [M, N] on every rank (one all-gather)."""
    P, _ = _world(group)
    M = y_local.shape[0]
    if P == 1:
        return y_local[:, :N]
    buf = torch.empty((P * M, w), dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(buf, y_local.contiguous(), group=group)
    if M == 1:
        return buf.view(1, P * w)[:, :N]
    return buf.view(P, M, w).permute(1, 0, 2).reshape(M, P * w)[:, :N]


class CudaBackend:
    """The single-GPU kernels of this package."""

    def gptq_matmul(self, x, qweight, qzeros, scales, K, N, gs, bits, zoff, x_perm=None):
        return _gptq_matmul(x, qweight, qzeros, scales, K, N, gs, bits, zoff, x_perm=x_perm)

    def q4k_matmul(self, x, raw, K, N):
        from .ggml import ggml_matmul
        return ggml_matmul(x, raw, "Q4_K", K, N)

    def route(self, logits, top_k, norm):
        r = _moe.route(logits, top_k, norm)
        return r.topk_idx, r.topk_w

    def group(self, ids, G, tile_rows=_moe.TILE_ROWS):
        """Sorted order of `ids` (values in [0, G)): (grouping, counts[G], row_src[n], pos_of[n])."""
        n = ids.numel()
        r = _moe.Routing(n, G, 1, ids.device, tile_rows)
        ids = ids.to(torch.int32).contiguous()
        _ffi.call("ql_moe_group", _ffi.ptr(ids), n, G, tile_rows, _ffi.ptr(r.counts), _ffi.ptr(r.offsets),
                  _ffi.ptr(r.cursor), _ffi.ptr(r.active), _ffi.ptr(r.n_active), _ffi.ptr(r.tiles),
                  _ffi.ptr(r.n_tiles), r.max_tiles, _ffi.ptr(r.row_token), _ffi.ptr(r.pair_row.view(-1)),
                  _ffi.stream_ptr())
        return r, r.counts, r.row_token[:n], r.pair_row.view(-1)[:n]

    def expert_ffn(self, x, row_src, grouping, gate_up, down, I):
        """down(silu(gate(x)) * up(x)) for the rows x[row_src[p]] in expert-sorted order p
        (grouping from `group`); returns [n, H] in that sorted order."""
        y = _moe.grouped_matmul(x, row_src, grouping, gate_up)
        return _moe.down_swiglu(y, grouping, down)

    def combine(self, z, pos_of, topk_w, T, k, H):
        out = torch.empty((T, H), dtype=torch.float32, device=z.device)
        pos = pos_of.to(torch.int32).contiguous()
        w = topk_w.to(torch.float32).contiguous()
        _ffi.call("ql_moe_combine", _ffi.ptr(z), _ffi.ptr(pos), _ffi.ptr(w), T, k, H, None, 0, None, 0,
                  _ffi.ptr(out), _ffi.dtype_code(out.dtype), out.stride(0), _ffi.stream_ptr())
        return out


class ShardedQuantizedLinear(torch.nn.Module):
    """GPTQ linear split by output columns over the ranks of `group`; forward returns the full
    [..., N] output on every rank (webtorch/_core.py:4446-4456 semantics)."""

    def __init__(self, qweight, qzeros, scales, bias, K, N, gs, bits, zero_offset=1.0, x_perm=None, group=None,
                 device=None, backend=None):
        super().__init__()
        self.group = group
        P, r = _world(group)
        self.K, self.N, self.gs, self.bits, self.zero_offset = int(K), int(N), int(gs), int(bits), float(zero_offset)
        self.backend = backend or CudaBackend()
        per = 32 // self.bits
        n0, n1, w = shard_range(self.N, P, r)
        self.n0, self.n1, self.w = n0, n1, w
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        qw = _to_dev(qweight, torch.int32, dev)[:, n0:n1]
        qz = _to_dev(qzeros, torch.int32, dev)[:, n0 // per:n1 // per]
        sc = _scale_tensor(scales, dev)[:, n0:n1]
        pad = w - (n1 - n0)
        if pad:   # zero weights (scale 0) in the padded tail columns
            qw = torch.nn.functional.pad(qw, (0, pad))
            qz = torch.nn.functional.pad(qz, (0, pad // per))
            sc = torch.nn.functional.pad(sc, (0, pad))
        self.register_buffer("qweight", qw.contiguous())
        self.register_buffer("qzeros", qz.contiguous())
        self.register_buffer("scales", sc.contiguous())
        self.register_buffer("x_perm", None if x_perm is None else _to_dev(x_perm, torch.int32, dev))
        self.register_buffer("bias", None if bias is None else _to_dev(bias, torch.float32, dev))

    @staticmethod
    def from_quantized(ql, group=None, backend=None):
        """Shard an existing (full) QuantizedLinear-like layer: qweight/qzeros/scales, Kp, Np, gs,
        bits, zero_offset, x_perm, bias (padding Kp/Np as the layer has it)."""
        m = ShardedQuantizedLinear(ql.qweight, ql.qzeros, ql.scales, ql.bias, ql.Kp, ql.Np, ql.gs, ql.bits,
                                   ql.zero_offset, x_perm=getattr(ql, "x_perm", None), group=group,
                                   device=ql.qweight.device, backend=backend)
        m.Kt, m.Nt = ql.Kt, ql.Nt
        return m

    def forward_local(self, x2d):
        """This rank's [M, w] slice."""
        return self.backend.gptq_matmul(x2d, self.qweight, self.qzeros, self.scales, self.K, self.w, self.gs,
                                        self.bits, self.zero_offset, self.x_perm)

    def forward(self, x):
        lead = x.shape[:-1]
        Kt = getattr(self, "Kt", self.K)
        Nt = getattr(self, "Nt", self.N)
        x2d = x.reshape(-1, Kt)
        if self.K != Kt:
            x2d = torch.nn.functional.pad(x2d, (0, self.K - Kt))
        y = _gather_columns(self.forward_local(x2d), self.w, self.N, self.group)[:, :Nt]
        if self.bias is not None:
            y = y + self.bias[:Nt]
        return y.reshape(*lead, Nt)


class ShardedGGMLLinear(torch.nn.Module):
    """Q4_K linear split by weight rows (output columns) over the ranks of `group`."""

    def __init__(self, raw, K, N, bias=None, group=None, device=None, backend=None):
        super().__init__()
        self.group = group
        P, r = _world(group)
        self.K, self.N = int(K), int(N)
        self.backend = backend or CudaBackend()
        n0, n1, w = shard_range(self.N, P, r, align=8)
        self.n0, self.n1, self.w = n0, n1, w
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        rows = _to_dev(raw, torch.uint8, dev).reshape(self.N, -1)[n0:n1]
        if w > n1 - n0:   # zero blocks (d = dmin = 0) decode to zero weights
            rows = torch.cat([rows, torch.zeros((w - (n1 - n0), rows.shape[1]), dtype=torch.uint8, device=dev)])
        self.register_buffer("raw", rows.contiguous())
        self.register_buffer("bias", None if bias is None else _to_dev(bias, torch.float32, dev))

    def forward(self, x):
        lead = x.shape[:-1]
        x2d = x.reshape(-1, self.K)
        y = _gather_columns(self.backend.q4k_matmul(x2d, self.raw, self.K, self.w), self.w, self.N, self.group)
        if self.bias is not None:
            y = y + self.bias
        return y.reshape(*lead, self.N)


class ExpertParallelMoE(torch.nn.Module):
    """Expert-parallel MoE block (lm_engine.moe_mlp semantics, webtorch/lm_engine.py:294-321).

    gate_up / down: this rank's StackedExperts (experts [r * E/P, (r + 1) * E/P)), or any objects
    the backend's expert_ffn accepts. `router` maps x [T, H] -> logits [T, E] (replicated)."""

    def __init__(self, router, gate_up, down, E, H, I, top_k, norm_topk_prob=True, group=None, backend=None):
        super().__init__()
        self.group = group
        self.P, self.r = _world(group)
        if E % self.P:
            raise ValueError("the expert count %d must divide over %d ranks" % (E, self.P))
        self.router, self.gate_up, self.down = router, gate_up, down
        self.E, self.H, self.I, self.top_k, self.norm = E, H, I, int(top_k), bool(norm_topk_prob)
        self.Ep = E // self.P
        self.backend = backend or CudaBackend()

    def _tile_rows(self, n):
        """Tile height for grouping n received rows over the local experts (CUDA backend)."""
        if not isinstance(self.backend, CudaBackend):
            return _moe.TILE_ROWS
        return _moe.tile_rows_for(n, self.Ep, self.H, getattr(self.gate_up, "gs", 128), n)

    def _all_to_all(self, out_rows, rows, out_splits, in_splits):
        if self.P == 1:
            return rows
        dist.all_to_all_single(out_rows, rows, out_splits, in_splits, group=self.group)
        return out_rows

    def forward(self, x):
        be = self.backend
        T, H = x.shape
        k = self.top_k
        logits = self.router(x)
        topk_idx, topk_w = be.route(logits, k, self.norm)
        flat = topk_idx.reshape(-1).to(torch.int32)
        dest = torch.div(flat, self.Ep, rounding_mode="floor").to(torch.int32)
        # 1. pairs grouped by destination rank (stable within a rank: atomics give an arbitrary
        #    order, which no output depends on)
        _, send_counts, row_src, pos_of = be.group(dest, self.P)
        send_x = x[torch.div(row_src.long(), k, rounding_mode="floor")]
        send_e = (flat[row_src.long()] - dest[row_src.long()] * self.Ep).to(torch.int32)
        # 2. counts, then rows and local expert ids
        recv_counts = torch.empty_like(send_counts)
        if self.P == 1:
            recv_counts = send_counts
        else:
            dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        n_recv = int(sum(rc))
        recv_x = self._all_to_all(torch.empty((n_recv, H), dtype=x.dtype, device=x.device), send_x, rc, sc)
        recv_e = self._all_to_all(torch.empty((n_recv,), dtype=torch.int32, device=x.device), send_e, rc, sc)
        # 3. local grouped expert FFN over the received rows
        grouping, _, lsrc, lpos = be.group(recv_e, self.Ep, self._tile_rows(n_recv))
        z_sorted = be.expert_ffn(recv_x, lsrc, grouping, self.gate_up, self.down, self.I)
        z_recv = z_sorted[lpos.long()]
        # 4. results back to the source ranks, in the order they were sent
        back = self._all_to_all(torch.empty((T * k, H), dtype=z_recv.dtype, device=x.device),
                                z_recv.contiguous(), sc, rc)
        return be.combine(back, pos_of, topk_w, T, k, H)
