"""Sharded linears and the expert-parallel MoE block on 2 GPUs (NCCL), one process per GPU, each
compared with the single-GPU operator on the same weights. Skipped with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest
import torch

from conftest import max_rel_err

pytestmark = pytest.mark.gpu
WORLD = 2
TOL = 2e-3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(rank, port, q):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        _checks(rank, dev)
        q.put((rank, None))
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc()))
    finally:
        torch.cuda.synchronize()
        dist.destroy_process_group()


def _checks(rank, dev):
    from webpytorch_b200 import moe, synth
    from webpytorch_b200.ggml import GGMLLinear
    from webpytorch_b200.qlinear import QuantizedLinear
    from webpytorch_b200.shard import ExpertParallelMoE, ShardedGGMLLinear, ShardedQuantizedLinear

    # GPTQ: decode (GEMV) and prefill (tcgen05 GEMM) through the sharded layer
    for (K, N, bits, M) in [(4096, 11008, 4, 1), (4096, 4864, 8, 16), (1024, 3000, 4, 256)]:
        w = synth.gptq_weights(K, N, bits, 128, seed=N + bits)
        full = QuantizedLinear.from_autogptq(w["qweight"], w["qzeros"], w["scales"], None, 128, bits, device=dev)
        sh = ShardedQuantizedLinear.from_quantized(full)
        x = torch.from_numpy(synth.activations(M, K, np.float16, seed=M)).to(dev)
        ref = full(x)
        got = sh(x)
        assert got.shape == ref.shape
        assert max_rel_err(got.cpu().numpy(), ref.cpu().numpy()) < TOL, (K, N, bits, M)

    # Q4_K rows
    N, K = 1000, 2048
    raw = synth.q4k_weights(N, K, seed=5)
    full = GGMLLinear(raw, "Q4_K", K, N, device=dev)
    sh = ShardedGGMLLinear(torch.from_numpy(raw), K, N, device=dev)
    x = torch.from_numpy(synth.activations(3, K, np.float32, seed=6)).to(dev)
    assert max_rel_err(sh(x).cpu().numpy(), full(x).cpu().numpy()) < TOL

    # expert parallel MoE vs the single-GPU block on the same experts (each rank its own tokens)
    E, k, H, I = 16, 4, 1024, 256
    exps = synth.moe_experts(E, H, I, bits=4, gs=128, seed=9)
    experts = [{p: QuantizedLinear.from_autogptq(e[p]["qweight"], e[p]["qzeros"], e[p]["scales"], None, 128, 4,
                                                 device=dev) for p in ("gate", "up", "down")} for e in exps]
    Ep = E // WORLD
    local = experts[rank * Ep:(rank + 1) * Ep]
    gu = moe.StackedExperts(local, ("gate", "up"), dev)
    dn = moe.StackedExperts(local, ("down",), dev)
    for T in (3, 300):
        g = torch.Generator(device=dev)
        g.manual_seed(100 * T + rank)
        logits = torch.randn((T, E), device=dev, generator=g)
        x = torch.randn((T, H), device=dev, generator=g).to(torch.bfloat16)
        single = moe.MoEBlock(lambda t: logits, experts, k)
        ep = ExpertParallelMoE(lambda t: logits, gu, dn, E, H, I, k)
        ref = single(x)
        got = ep(x)
        assert max_rel_err(got.cpu().numpy(), ref.cpu().numpy()) < TOL, T


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_sharded_operators_on_two_gpus():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(WORLD)]
    for p in procs:
        p.join(timeout=120)
    bad = [e for _, e in res if e]
    assert not bad, "\n".join(bad)
