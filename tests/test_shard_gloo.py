"""Multi-process (world size 2, gloo on CPU) tests of the sharded linears and the
expert-parallel MoE block. The collective choreography of webpytorch_b200/shard.py runs
unchanged; the per-rank compute is the numpy oracle standing in for the CUDA kernels (a CPU
backend defined here), so these check partitioning, padding, exchange order and combine."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import gptq as og
from oracle import moe as om
from oracle import q4k as oq
from webpytorch_b200 import synth

WORLD = 2


class OracleBackend:
    """CPU compute with the oracle: the stand-in for shard.CudaBackend in these tests."""

    def gptq_matmul(self, x, qweight, qzeros, scales, K, N, gs, bits, zoff, x_perm=None):
        xf = x.float().numpy()
        if x_perm is not None:
            xf = xf[:, x_perm.numpy()]
        y = og.gptq_matmul(xf, qweight.numpy().view(np.int32), qzeros.numpy().view(np.int32),
                           scales.numpy(), K, N, gs, bits, zoff)
        return torch.from_numpy(np.ascontiguousarray(y, dtype=np.float32))

    def q4k_matmul(self, x, raw, K, N):
        W = oq.dequant(raw.numpy().reshape(-1), N * K).reshape(N, K)
        return torch.from_numpy((x.float().numpy().astype(np.float64) @ W.T.astype(np.float64)).astype(np.float32))

    def route(self, logits, top_k, norm):
        idx, w = om.route(logits.numpy(), top_k, norm)
        return torch.from_numpy(idx.astype(np.int32)), torch.from_numpy(w.astype(np.float32))

    def group(self, ids, G, tile_rows=128):
        ids = ids.numpy()
        row_src = np.argsort(ids, kind="stable").astype(np.int32)
        pos_of = np.empty_like(row_src)
        pos_of[row_src] = np.arange(len(ids), dtype=np.int32)
        counts = np.bincount(ids, minlength=G).astype(np.int32)
        sorted_ids = ids[row_src]
        return sorted_ids, torch.from_numpy(counts), torch.from_numpy(row_src), torch.from_numpy(pos_of)

    def expert_ffn(self, x, row_src, sorted_ids, gate_up, down, I):
        xs = x.float().numpy()[row_src.numpy()]
        out = np.zeros((len(xs), down[0]["N"]), np.float32)
        for e in np.unique(sorted_ids):
            rows = np.nonzero(sorted_ids == e)[0]
            g = gate_up[e]
            d = down[e]
            y = og.quantized_linear(xs[rows], g["qweight"], g["qzeros"], g["scales"], None, g["K"], g["N"],
                                    g["K"], g["N"], g["gs"], g["bits"], 1.0)
            a = om.silu(y[:, :I]) * y[:, I:]
            out[rows] = og.quantized_linear(a, d["qweight"], d["qzeros"], d["scales"], None, d["K"], d["N"],
                                            d["K"], d["N"], d["gs"], d["bits"], 1.0)
        return torch.from_numpy(out)

    def combine(self, z, pos_of, topk_w, T, k, H):
        z = z.numpy()
        pos = pos_of.numpy().reshape(T, k)
        w = topk_w.numpy().reshape(T, k)
        return torch.from_numpy(np.einsum("tk,tkh->th", w, z[pos]).astype(np.float32))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(rank, port, fn, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        fn(rank)
        q.put((rank, None))
    except Exception as e:   # reported to the parent
        import traceback
        q.put((rank, traceback.format_exc()))
    finally:
        dist.destroy_process_group()


def _spawn(fn):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, port, fn, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    errs = [q.get(timeout=300) for _ in range(WORLD)]
    for p in procs:
        p.join(timeout=60)
    bad = [e for _, e in errs if e]
    assert not bad, "\n".join(bad)


def _gptq_case(rank):
    from webpytorch_b200.shard import ShardedQuantizedLinear, shard_range
    for (K, N, bits, M) in [(256, 200, 4, 1), (384, 96, 8, 3), (128, 72, 4, 5)]:
        w = synth.gptq_weights(K, N, bits, 128 if K % 128 == 0 else 32, seed=K + N)
        gs = 128 if K % 128 == 0 else 32
        x = synth.activations(M, K, np.float32, seed=7)
        m = ShardedQuantizedLinear(torch.from_numpy(w["qweight"]), torch.from_numpy(w["qzeros"]),
                                   torch.from_numpy(w["scales"]), None, K, N, gs, bits, 1.0, device="cpu",
                                   backend=OracleBackend())
        n0, n1, width = shard_range(N, WORLD, rank)
        assert m.qweight.shape == (K // (32 // bits), width)
        y = m(torch.from_numpy(x)).numpy()
        ref = og.gptq_matmul(x, w["qweight"], w["qzeros"], w["scales"], K, N, gs, bits, 1.0)
        assert y.shape == (M, N)
        np.testing.assert_allclose(y, ref, rtol=1e-6, atol=1e-6)


def _q4k_case(rank):
    from webpytorch_b200.shard import ShardedGGMLLinear
    N, K, M = 40, 512, 2
    raw = synth.q4k_weights(N, K, seed=3)
    x = synth.activations(M, K, np.float32, seed=4)
    m = ShardedGGMLLinear(torch.from_numpy(raw), K, N, device="cpu", backend=OracleBackend())
    y = m(torch.from_numpy(x)).numpy()
    W = oq.dequant(raw.reshape(-1), N * K).reshape(N, K)
    np.testing.assert_allclose(y, (x.astype(np.float64) @ W.T.astype(np.float64)).astype(np.float32),
                               rtol=1e-5, atol=1e-5)


def _moe_case(rank):
    from webpytorch_b200.shard import ExpertParallelMoE
    E, k, H, I = 8, 2, 128, 64
    exps = synth.moe_experts(E, H, I, bits=4, gs=64, seed=11)

    def pack(w, Kin, Nout):
        return dict(w, K=Kin, N=Nout, gs=64, bits=4)
    gate_up = {}
    down = {}
    Ep = E // WORLD
    for e in range(rank * Ep, (rank + 1) * Ep):
        g, u = exps[e]["gate"], exps[e]["up"]
        gate_up[e - rank * Ep] = pack({"qweight": np.concatenate([g["qweight"], u["qweight"]], 1),
                                       "qzeros": np.concatenate([g["qzeros"], u["qzeros"]], 1),
                                       "scales": np.concatenate([g["scales"], u["scales"]], 1)}, H, 2 * I)
        down[e - rank * Ep] = pack(exps[e]["down"], I, H)
    T = 5 + 3 * rank          # different token counts per rank
    rng = np.random.default_rng(100 + rank)
    logits = rng.standard_normal((T, E)).astype(np.float32)
    x = rng.standard_normal((T, H)).astype(np.float32)
    blk = ExpertParallelMoE(lambda t: torch.from_numpy(logits), gate_up, down, E, H, I, k,
                            backend=OracleBackend())
    y = blk(torch.from_numpy(x)).numpy()

    def lin(w, Kin, Nout):
        return lambda v: og.quantized_linear(v, w["qweight"], w["qzeros"], w["scales"], None, Kin, Nout, Kin, Nout,
                                             64, 4, 1.0)
    ref = om.moe_mlp(x, logits, [(lin(e["gate"], H, I), lin(e["up"], H, I), lin(e["down"], I, H)) for e in exps], k)
    np.testing.assert_allclose(y, ref, rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("case", [_gptq_case, _q4k_case, _moe_case])
def test_two_ranks_gloo(case):
    _spawn(case)


def test_shard_range_covers_all_columns():
    from webpytorch_b200.shard import shard_range
    for N in (4096, 11008, 18944, 200, 32):
        for P in (1, 2, 4, 8):
            cols = []
            for r in range(P):
                n0, n1, w = shard_range(N, P, r)
                assert w % 32 == 0 and n1 - n0 <= w
                cols.extend(range(n0, n1))
            assert cols == list(range(N))
