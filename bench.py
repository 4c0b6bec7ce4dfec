"""Benchmark of the B200 quantized-linear hot path (one JSON line on rank 0).

Headline (config 1): int4 GPTQ decode GEMV at M=1 over the five (K, N)
shapes {(4096,4096), (4096,11008), (11008,4096), (4096,14336), (14336,4096)}, group 128,
fp16 x, fp32 out. One step = one pass over the five shapes on each of R=4 distinct weight
copies (20 GEMVs, 466 MB of packed weights > 2 x L2), so no launch finds its weights in L2.
`value` = algorithmic bytes (packed weights + scales + zeros + x + out) / device time, inputs
resident in HBM. `e2e` = the same bytes through the public Python operator with pinned host
x copied in and y copied out every step.

N > 1 (torchrun): every rank holds the column shard of layers N times wider (its shard has
the 1-GPU shape, so per-rank work is fixed: weak scaling) and each step ends with one NCCL
all-gather of the step's 20 outputs; value = all ranks' bytes / max time over ranks. The
`moe_ep` section runs config 4 expert-parallel (128 / N experts per rank, T tokens per rank).

--impl reference: the reference's CPU algorithm (the numpy port in oracle/, the reference
package itself cannot travel) on a bounded sample of the same workload, same metric.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SHAPES = [(4096, 4096), (4096, 11008), (11008, 4096), (4096, 14336), (14336, 4096)]
GS = 128
COPIES = 4
METRIC = "int4 GEMV HBM GB/s at M=1 (config 1 sweep)"
GEMM_SHAPES = [(4096, 11008), (3584, 18944)]
GEMM_MS = (128, 512, 2048)
GEMM_M = 2048
L2_BYTES = 126 * 2 ** 20
# DRAM bytes per launch of gptq_gemv_tma_kernel over its algorithmic bytes, from one ncu capture
# (dram__bytes_read.sum + dram__bytes_write.sum = 30.606 MB for the K=4096, N=14336 launch whose
# algorithmic bytes are 30.906 MB); traffic grows with the weight bytes, so it scales per shape
GEMV_TRAFFIC_RATIO = 30.606 / 30.906


def gemv_bytes(K, N, M=1, bits=4, gs=GS, x_bytes=2, out_bytes=4):
    """Algorithmic bytes of one GEMV: packed weights + scales(fp16) + zeros + x + out."""
    per = 32 // bits
    w = K * N * bits // 8 + (K // gs) * N * 2 + (K // gs) * (N // per) * 4
    return w + M * K * x_bytes + M * N * out_bytes


def step_bytes():
    return COPIES * sum(gemv_bytes(K, N) for K, N in SHAPES)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as fh:
            d = json.load(fh)
        return float(d["hbm_gbs"]), float(d.get("bf16_tflops", 1590.0)), "measured"
    return 6650.0, 1590.0, "fallback"


MOE_E, MOE_TOPK, MOE_H, MOE_I = 128, 8, 2048, 768
MOE_TOKENS = (1, 32, 256, 2048)
Q4K_K, Q4K_N, Q4K_MS, Q4K_COPIES = 4096, 14336, (1, 8, 16, 64, 512), 8


def rand_gptq(K, N, dev, g, E=None, bits=4):
    """Config-0 distributions on the device: uniform packed words, fp16 scales U[0.002, 0.02]."""
    per = 32 // bits
    lead = () if E is None else (E,)
    qw = torch_mod().randint(-2 ** 31, 2 ** 31 - 1, lead + (K // per, N), dtype=torch_mod().int32, device=dev,
                             generator=g)
    qz = torch_mod().randint(-2 ** 31, 2 ** 31 - 1, lead + (K // GS, N // per), dtype=torch_mod().int32,
                             device=dev, generator=g)
    sc = (torch_mod().rand(lead + (K // GS, N), device=dev, generator=g) * 0.018 + 0.002).half()
    return qw, qz, sc


def rand_q4k(N, K, dev, g):
    """Config-2 super-blocks on the device: uniform bytes, then fp16 d and dmin U[1e-3, 1e-2]."""
    torch = torch_mod()
    nb = N * (K // 256)
    raw = torch.randint(0, 256, (nb, 144), dtype=torch.uint8, device=dev, generator=g)
    dd = (torch.rand((nb, 2), device=dev, generator=g) * 9e-3 + 1e-3).half()
    raw[:, 0:4] = dd.view(torch.uint8).reshape(nb, 4)
    return raw.reshape(N, (K // 256) * 144).contiguous()


def torch_mod():
    import torch
    return torch


def event_time(fn, reps):
    """Average device ms of fn() over reps calls (CUDA events on the current stream)."""
    torch = torch_mod()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def bench_moe(dev, g, hbm, bf16_peak):
    """Config 4: Qwen3-MoE-shaped block (128 experts, top-8, H=2048, I=768, int4 g128, bf16 x).
    Each timed step is a CUDA graph over L independent layers (own experts, logits and x) so
    that the active experts' weights come from HBM, not L2."""
    torch = torch_mod()
    from webpytorch_b200 import moe
    out = {}
    for T in MOE_TOKENS:
        L = 8 if T <= 256 else 2
        layers = []
        for _ in range(L):
            gu = moe.StackedExperts.from_packed(*rand_gptq(MOE_H, 2 * MOE_I, dev, g, E=MOE_E), GS, 4)
            dn = moe.StackedExperts.from_packed(*rand_gptq(MOE_I, MOE_H, dev, g, E=MOE_E), GS, 4)
            logits = torch.randn((T, MOE_E), device=dev, generator=g)
            blk = moe.MoEBlock.from_stacked(lambda t, _l=logits: _l, gu, dn, MOE_TOPK)
            x = torch.randn((T, MOE_H), device=dev, generator=g).to(torch.bfloat16)
            layers.append((blk, x, logits))
        act = sum(int(torch.topk(lg, MOE_TOPK, dim=1).indices.unique().numel()) for _, _, lg in layers)

        def fwd():
            for blk, x, _ in layers:
                blk(x)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(3):
                fwd()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=s):
                fwd()
        torch.cuda.current_stream().wait_stream(s)
        for _ in range(3):
            gr.replay()
        reps = 50 if T <= 256 else 10
        ms = event_time(gr.replay, reps) / L
        exp_bytes = layers[0][0].gate_up.expert_nbytes() + layers[0][0].down.expert_nbytes()
        wbytes = act / L * exp_bytes
        flops = 2.0 * T * MOE_TOPK * (MOE_H * 2 * MOE_I + MOE_I * MOE_H)
        r = {"us": round(ms * 1e3, 2), "tokens/s": round(T / (ms / 1e3), 1),
             "active_experts": round(act / L, 2), "expert_GB/s": round(wbytes / (ms / 1e3) / 1e9, 1),
             "expert_frac_of_hbm": round(wbytes / (ms / 1e3) / 1e9 / hbm, 4),
             "TFLOP/s": round(flops / (ms / 1e3) / 1e12, 1),
             "frac_of_bf16_peak": round(flops / (ms / 1e3) / 1e12 / bf16_peak, 4), "layers_per_graph": L}
        out["T%d" % T] = r
        del gr, layers
        torch.cuda.empty_cache()
    return out


def bench_moe_ep(dev, g, world, timed):
    """Config 4 across `world` GPUs, expert parallel: each rank holds 128 / world experts, routes
    its own T tokens (weak scaling in tokens) and exchanges rows with two all-to-alls per layer.
    Timed eagerly (the dispatch sizes are read back to the host every layer), max over ranks."""
    torch = torch_mod()
    from webpytorch_b200 import moe
    from webpytorch_b200.shard import ExpertParallelMoE
    Ep = MOE_E // world
    out = {}
    for T in (32, 256, 2048):
        L = 4
        layers = []
        for _ in range(L):
            gu = moe.StackedExperts.from_packed(*rand_gptq(MOE_H, 2 * MOE_I, dev, g, E=Ep), GS, 4)
            dn = moe.StackedExperts.from_packed(*rand_gptq(MOE_I, MOE_H, dev, g, E=Ep), GS, 4)
            logits = torch.randn((T, MOE_E), device=dev, generator=g)
            x = torch.randn((T, MOE_H), device=dev, generator=g).to(torch.bfloat16)
            layers.append((ExpertParallelMoE(lambda t, _l=logits: _l, gu, dn, MOE_E, MOE_H, MOE_I, MOE_TOPK), x))

        def fwd():
            for blk, x in layers:
                blk(x)
        for _ in range(2):
            fwd()
        reps = 5
        ms, _, _ = timed(lambda: [fwd() for _ in range(reps)], 1)
        ms_layer = ms / (reps * L)
        out["T%d_per_rank" % T] = {"us_per_layer": round(ms_layer * 1e3, 2),
                                   "tokens/s": round(T * world / (ms_layer / 1e3), 1),
                                   "experts_per_rank": Ep, "tokens_per_rank": T}
        del layers
        torch.cuda.empty_cache()
    return out


def bench_q4k(dev, g, hbm):
    """Config 2: Q4_K dequant-GEMV/GEMM, K=4096, N=14336, fp32 x, M in Q4K_MS; rotating copies."""
    torch = torch_mod()
    from webpytorch_b200.ggml import ggml_matmul
    raws = [rand_q4k(Q4K_N, Q4K_K, dev, g) for _ in range(Q4K_COPIES)]
    res = {}
    for M in Q4K_MS:
        x = torch.randn((M, Q4K_K), device=dev, generator=g)
        y = torch.empty((M, Q4K_N), device=dev)

        def run():
            for r in raws:
                ggml_matmul(x, r, "Q4_K", Q4K_K, Q4K_N, out=y)
        gr = torch.cuda.CUDAGraph()
        run()
        torch.cuda.synchronize()
        with torch.cuda.graph(gr):
            run()
        for _ in range(3):
            gr.replay()
        ms = event_time(gr.replay, 20) / Q4K_COPIES
        nbytes = raws[0].numel() + M * Q4K_K * 4 + M * Q4K_N * 4
        res["M%d" % M] = {"us": round(ms * 1e3, 2), "GB/s": round(nbytes / (ms / 1e3) / 1e9, 1),
                          "frac_of_hbm": round(nbytes / (ms / 1e3) / 1e9 / hbm, 4)}
        del gr
    return res


DEC_CFG = {"H": 3584, "NH": 28, "NKV": 4, "HD": 128, "I": 18944, "L": 28, "pos": 512, "lmax": 1024}


def bench_decode(dev, g, hbm, steps=50):
    """The decode step (8(f) row 1) on a synthetic Qwen2.5-7B-shaped stack: 28 layers of H=3584,
    28 query / 4 key-value heads of 128, SwiGLU I=18944, int4 g128 AutoGPTQ weights with q/k/v
    biases, KV cache filled up to position 512; one graph replay per token (5 launches a layer)."""
    torch = torch_mod()
    from webpytorch_b200.decode import DecodeLayer, DecodeStack
    from webpytorch_b200.qlinear import QuantizedLinear
    c = DEC_CFG
    H, NH, NKV, HD, I, L = c["H"], c["NH"], c["NKV"], c["HD"], c["I"], c["L"]

    def lin(K, N, bias=False):
        qw, qz, sc = rand_gptq(K, N, dev, g)
        b = torch.randn(N, device=dev, generator=g) * 0.1 if bias else None
        return QuantizedLinear(qw, qz, sc, b, K, N, K, N, GS, 4, zero_offset=1.0, device=dev)
    layers = []
    for _ in range(L):
        layers.append(DecodeLayer(lin(H, NH * HD, True), lin(H, NKV * HD, True), lin(H, NKV * HD, True),
                                  lin(NH * HD, H), lin(H, I), lin(H, I), lin(I, H),
                                  torch.rand(H, device=dev, generator=g) + 0.5,
                                  torch.rand(H, device=dev, generator=g) + 0.5))
    stack = DecodeStack(layers, H, NH, NKV, HD, c["lmax"])
    for kc, vc in zip(stack.kc, stack.vc):   # a context of `pos` earlier tokens
        kc.normal_(generator=g)
        vc.normal_(generator=g)
    emb = torch.randn(H, device=dev, generator=g)
    for _ in range(3):
        stack.step(emb, c["pos"])
    torch.cuda.synchronize()
    ms = event_time(stack.graph.replay, steps)
    wbytes = sum(l.nbytes() for l in layers)
    kv = L * 2 * NKV * (c["pos"] + 1) * HD * 4
    return {"workload": "synthetic Qwen2.5-7B-shaped decode stack: %d layers, H=%d, heads %d/%d x %d, I=%d, int4 "
                        "g128, context position %d, one CUDA-graph replay per token (%d launches)"
                        % (L, H, NH, NKV, HD, I, c["pos"], stack.launches_per_step()),
            "ms_per_token": round(ms, 4), "tokens/s": round(1e3 / ms, 1),
            "weight_MB_per_token": round(wbytes / 1e6, 1), "kv_MB_per_token": round(kv / 1e6, 1),
            "GB/s": round((wbytes + kv) / (ms / 1e3) / 1e9, 1),
            "frac_of_hbm": round((wbytes + kv) / (ms / 1e3) / 1e9 / hbm, 4)}


def profile_case(name):
    """A small, fixed launch sequence of one kernel for `ncu` (few launches, a few GB at most;
    inputs larger than L2 where the kernel streams weights)."""
    torch = torch_mod()
    from webpytorch_b200 import _ffi
    from webpytorch_b200.qlinear import QuantizedLinear, _gptq_matmul
    dev = torch.device("cuda", 0)
    _ffi.load(build_if_missing=False)
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    if name in ("gemv", "gemv_narrow"):      # gptq_gemv_tma_kernel, M=1, 6 copies (> L2)
        K, N = (4096, 14336) if name == "gemv" else (14336, 4096)   # 256- / 128-column tiles
        ws = [rand_gptq(K, N, dev, g) for _ in range(6)]
        x = torch.randn((1, K), device=dev, generator=g).half()
        y = torch.empty((1, N), device=dev)
        for qw, qz, sc in ws:
            _gptq_matmul(x, qw, qz, sc, K, N, GS, 4, 1.0, out=y)
    elif name == "gemm":                     # prep_x_kernel + gptq_gemm_tc_kernel, config 3 shape 1
        K, N, M = 4096, 11008, 2048
        qw, qz, sc = rand_gptq(K, N, dev, g)
        gidx = (torch.arange(K, device=dev) // GS)[torch.randperm(K, device=dev, generator=g)]
        ql = QuantizedLinear.from_autogptq(qw, qz, sc, None, GS, 4, g_idx=gidx, device=dev)
        x = torch.randn((M, K), device=dev, generator=g).to(torch.bfloat16)
        yb = torch.empty((M, N), device=dev, dtype=torch.bfloat16)
        for _ in range(3):
            ql(x, out=yb, out_dtype=torch.bfloat16)
    elif name in ("moe_decode", "moe_prefill"):   # config 4, T = 32 (grouped GEMV) / 2048 (grouped GEMM)
        from webpytorch_b200 import moe
        T = 32 if name == "moe_decode" else 2048
        gu = moe.StackedExperts.from_packed(*rand_gptq(MOE_H, 2 * MOE_I, dev, g, E=MOE_E), GS, 4)
        dn = moe.StackedExperts.from_packed(*rand_gptq(MOE_I, MOE_H, dev, g, E=MOE_E), GS, 4)
        logits = torch.randn((T, MOE_E), device=dev, generator=g)
        blk = moe.MoEBlock.from_stacked(lambda t: logits, gu, dn, MOE_TOPK)
        x = torch.randn((T, MOE_H), device=dev, generator=g).to(torch.bfloat16)
        for _ in range(2):
            blk(x)
    elif name in ("q4k", "q4k_m8", "q4k_m64"):   # config 2, 8 copies (264 MB): q4k_gemv_tma_kernel at M=1 / 8,
        from webpytorch_b200.ggml import ggml_matmul   # the tensor-core path (gptq_gemm_tc_kernel<Q4_K>) at M=64
        raws = [rand_q4k(Q4K_N, Q4K_K, dev, g) for _ in range(Q4K_COPIES)]
        M = {"q4k": 1, "q4k_m8": 8, "q4k_m64": 64}[name]
        x = torch.randn((M, Q4K_K), device=dev, generator=g)
        y = torch.empty((M, Q4K_N), device=dev)
        for r in raws:
            ggml_matmul(x, r, "Q4_K", Q4K_K, Q4K_N, out=y)
    elif name == "ggml_q6k":                 # ggml_gemv_kernel<Q6_K>, K=4096, N=14336, M=1, 8 copies (386 MB)
        from webpytorch_b200 import synth
        from webpytorch_b200.ggml import ggml_matmul
        raws = [torch.from_numpy(synth.ggml_weights("Q6_K", Q4K_N, Q4K_K, seed=i).reshape(-1)).to(dev)
                for i in range(8)]
        x = torch.randn((1, Q4K_K), device=dev, generator=g)
        for r in raws:
            ggml_matmul(x, r, "Q6_K", Q4K_K, Q4K_N)
    elif name in ("decode_attn", "decode_gateup"):   # decode-step kernels at the bench's 7B shape
        from webpytorch_b200.decode import DecodeLayer, DecodeStack, fused_linear
        c = DEC_CFG
        H, NH, NKV, HD, I = c["H"], c["NH"], c["NKV"], c["HD"], c["I"]

        def lin(K, N):
            qw, qz, sc = rand_gptq(K, N, dev, g)
            return QuantizedLinear(qw, qz, sc, None, K, N, K, N, GS, 4, zero_offset=1.0, device=dev)
        lays = [DecodeLayer(lin(H, NH * HD), lin(H, NKV * HD), lin(H, NKV * HD), lin(NH * HD, H), lin(H, I),
                            lin(H, I), lin(I, H), torch.ones(H, device=dev), torch.ones(H, device=dev))
                for _ in range(4)]
        st = DecodeStack(lays, H, NH, NKV, HD, c["lmax"], graph=False)
        for kc, vc in zip(st.kc, st.vc):
            kc.normal_(generator=g)
            vc.normal_(generator=g)
        st.step(torch.randn(H, device=dev, generator=g), c["pos"])
    else:
        raise SystemExit("unknown profile case %r" % name)
    torch.cuda.synchronize()
    rc = _ffi.load().ql_device_status()
    print(json.dumps({"profile_case": name, "device_status": rc}))
    return 1 if rc else 0


class ClockSampler:
    """SM clocks, power and throttle reasons sampled in the background during the timed region:
    through NVML every millisecond when pynvml is importable (the timed regions are a few ms),
    else with nvidia-smi. Read-only queries; no GPU setting is touched."""

    def __init__(self, index, period_ms=50):
        self.index, self.period_ms = index, period_ms
        self.samples = []
        self.proc = None
        self.nvml = None
        self.stop = False

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:   # the CUDA device's own GPU (CUDA ordinals and NVML indices can differ)
            pr = torch_mod().cuda.get_device_properties(self.index)
            bus = "%08x:%02x:%02x.0" % (pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId_v2(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def _poll(self):
        nv, h = self.nvml
        R = [nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
             nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap]
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        while not self.stop:
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                pw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                flags = ["Active" if rs & r else "Not Active" for r in R]
                self.samples.append((time.time(), ["", str(sm), str(mx), str(pw), hex(rs)] + flags))
            except Exception:
                return
            time.sleep(0.001)

    def __enter__(self):
        try:
            self.nvml = self._nvml_handle()
            self.th = threading.Thread(target=self._poll, daemon=True)
            self.th.start()
            return self
        except Exception:
            self.nvml = None
        q = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), "--query-gpu=" + q,
                                          "--format=csv,noheader,nounits", "-lms", str(self.period_ms)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.th = threading.Thread(target=self._read, daemon=True)
            self.th.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.samples.append((time.time(), parts))

    def mark(self):
        return time.time()

    def __exit__(self, *a):
        if self.nvml is not None:
            self.stop = True
            self.th.join(timeout=2)
            return
        if self.proc is not None:
            time.sleep(self.period_ms / 1000.0 * 2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self, t0, t1):
        def num(s):
            try:
                return float(s)
            except ValueError:
                return None
        inside = [p for (t, p) in self.samples if t0 <= t <= t1]
        window = "timed"
        if not inside:   # timed region shorter than the sampling period: nearest samples
            window = "nearest"
            inside = [p for (t, p) in sorted(self.samples, key=lambda s: abs(s[0] - (t0 + t1) / 2))[:3]]
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [num(p[1]) for p in inside if num(p[1]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for p in inside for i in range(4) if p[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": num(inside[0][2]),
                "reasons": reasons, "samples": len(inside), "window": window,
                "power_w_max": max((num(p[3]) or 0.0) for p in inside)}


def workload_config(world):
    """The `config` object of the JSON line; both arms (ours and --impl reference) print the same one."""
    return {"workload": "config1: int4 g128 GEMV M=1 over (K,N) in %s, fp16 x, fp32 out" % (SHAPES,),
            "bits": 4, "group_size": GS, "M": 1,
            "parallelism": ("N-sharded x%d: each rank holds the column shard (the 1-GPU shape) of layers "
                            "%d times wider; one NCCL all-gather of the step's outputs per step"
                            % (world, world)) if world > 1 else "single GPU",
            "l2": "inputs larger than L2 (rotating weight copies)"}


def _reference_gemv_sampler(rng):
    """Whole config-1 GEMVs (M=1, int4 g128), round-robin over the five shapes, through the
    step-for-step port of the reference's `_gptq_matmul_np` (oracle/gptq.py)."""
    from oracle import gptq as og
    from webpytorch_b200 import synth
    ws = {s: synth.gptq_weights(s[0], s[1], 4, GS, rng=rng) for s in SHAPES}
    xs = {K: synth.activations(1, K, np.float16, rng=rng) for K, _ in SHAPES}

    def one(i):
        K, N = SHAPES[i % len(SHAPES)]
        w = ws[(K, N)]
        og.gptq_matmul_np_steps(xs[K].astype(np.float32), w["qweight"], w["qzeros"], w["scales"], K, N, GS, 4, 1.0)
        return gemv_bytes(K, N)
    return one


def cpu_baseline(seconds=10.0):
    """The reference's CPU algorithm (the step-for-step numpy port of `_gptq_matmul_np`) on the
    host cores, whole config-1 GEMVs, for about `seconds`."""
    one = _reference_gemv_sampler(np.random.default_rng(0))
    one(0)
    t_end = time.perf_counter() + seconds
    done_bytes, busy, n = 0, 0.0, 0
    while time.perf_counter() < t_end or n == 0:
        t0 = time.perf_counter()
        done_bytes += one(n)
        busy += time.perf_counter() - t0
        n += 1
    return {"value": round(done_bytes / busy / 1e9, 4), "unit": "GB/s", "cores": os.cpu_count(),
            "kind": "port", "sample": "%d whole GEMVs (M=1, int4 g128, round-robin over the 5 config-1 shapes) "
                                      "through the step-for-step port of _gptq_matmul_np, %.1f s, numpy/OpenBLAS "
                                      "with all host threads" % (n, busy)}


def run_reference(args):
    """The reference arm: its CPU implementation of the path (the numpy port; the reference
    package itself is not on the GPU box) on the same workload and metric as our arm. One step
    is one whole config-1 GEMV (round-robin over the five shapes): a bounded sample of the
    step our arm times. Under torchrun only rank 0 runs."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    if rank != 0:
        return 0
    one = _reference_gemv_sampler(np.random.default_rng(0))
    for i in range(args.warmup):
        one(i)
    t0 = time.perf_counter()
    tot = 0
    for i in range(args.steps):
        tot += one(i)
    dt = time.perf_counter() - t0
    v = tot / dt / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int4 weights, fp32 x/out",
            "data": "synthetic", "config": workload_config(world),
            "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
                             "sample": "%d whole GEMVs (one per step, round-robin over the 5 config-1 shapes) "
                                       "through the step-for-step port of _gptq_matmul_np, %.1f s"
                                       % (args.steps, dt)},
            "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--skip-gemm", action="store_true")
    ap.add_argument("--skip-extra", action="store_true", help="skip the config-2 and config-4 sections")
    ap.add_argument("--profile", default=None,
                    help="run one small fixed case for ncu: gemv | gemv_narrow | gemm | moe_decode | "
                         "moe_prefill | q4k | q4k_m8 | q4k_m64 | ggml_q6k | decode_attn | decode_gateup")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.profile:
        return profile_case(args.profile)
    if args.impl == "reference":
        return run_reference(args)

    import torch
    import torch.distributed as dist

    from webpytorch_b200 import _ffi
    from webpytorch_b200.qlinear import _gptq_matmul

    # stdout carries exactly one JSON line (rank 0): anything libraries print there (NCCL's
    # version banner, for one) goes to stderr instead
    json_out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    _ffi.load(build_if_missing=False)

    # ---- synthetic weights (config-1 distributions), R copies per shape, generated on device
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    # Every GEMV writes its [1, N] output into one packed per-rank buffer. With N > 1 ranks each
    # rank holds the column shard of layers N times wider (its shard has the 1-GPU shape, weak
    # scaling) and a step ends with one all-gather of all 20 output slices.
    lay = []
    n_out = COPIES * sum(N for _, N in SHAPES)
    y_all = torch.empty((1, n_out), device=dev, dtype=torch.float32)
    gathered = torch.empty((world, n_out), device=dev, dtype=torch.float32) if world > 1 else None
    off = 0
    for c in range(COPIES):
        for (K, N) in SHAPES:
            qw, qz, sc = rand_gptq(K, N, dev, g)
            x = torch.randn((1, K), device=dev, generator=g).half()
            lay.append((K, N, qw, qz, sc, x, y_all[:, off:off + N]))
            off += N

    def launch(L):
        K, N, qw, qz, sc, x, y = L
        _gptq_matmul(x, qw, qz, sc, K, N, GS, 4, 1.0, out=y)

    def step():
        for L in lay:
            launch(L)
        if world > 1:
            dist.all_gather_into_tensor(gathered, y_all)

    # ---- capture one step into a CUDA graph (launch-bound otherwise), warm up first; a second
    # graph with programmatic dependent launch is timed for comparison.
    def capture(pdl):
        _ffi.set_launch_flags(_ffi.LAUNCH_PDL if pdl else 0)
        for _ in range(3):
            step()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            step()
        torch.cuda.synchronize()
        _ffi.set_launch_flags(0)
        return gr

    # plain launches are the headline: with this kernel's two resident CTAs per SM, programmatic
    # dependent launch places the next GEMV's CTAs unevenly and measures slower
    graph = capture(pdl=False)
    graph_pdl = capture(pdl=True)
    for _ in range(args.warmup):
        graph.replay()
        graph_pdl.replay()
    torch.cuda.synchronize()

    def timed(fn, n):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.time()
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        t1 = time.time()
        if world > 1:
            dist.barrier()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms, t0, t1

    sampler = ClockSampler(local)
    with sampler:
        time.sleep(0.15)
        ms, t0, t1 = timed(graph.replay, args.steps)
        clocks = sampler.summary(t0, t1)
    ms_pdl, _, _ = timed(graph_pdl.replay, args.steps)

    # ---- per-shape launch durations: a graph of 10 passes over >= 320 MB of one shape's
    # weight copies (each launch reads its weights from HBM), timed with CUDA events
    per_shape = {}
    for (K, N) in (SHAPES if world == 1 else []):
        Ls = [L for L in lay if (L[0], L[1]) == (K, N)]
        # rotate over at least 320 MB of this shape's weights so no launch finds them in L2
        extra = max(0, -(-320_000_000 // gemv_bytes(K, N)) - len(Ls))
        for _ in range(extra):
            qw, qz, sc = rand_gptq(K, N, dev, g)
            Ls.append((K, N, qw, qz, sc, Ls[0][5], Ls[0][6]))
        nl = 10 * len(Ls)
        res = {}
        for pdl in (False, True):
            _ffi.set_launch_flags(_ffi.LAUNCH_PDL if pdl else 0)
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                for i in range(nl):
                    launch(Ls[i % len(Ls)])
            _ffi.set_launch_flags(0)
            gr.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(3):
                gr.replay()
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (3 * nl)
            res["pdl" if pdl else "plain"] = us
            del gr
        del Ls
        per_shape["%dx%d" % (K, N)] = {"us": round(res["plain"], 3), "us_pdl": round(res["pdl"], 3),
                                       "GB/s": round(gemv_bytes(K, N) / res["plain"] / 1e3, 1),
                                       "GB/s_pdl": round(gemv_bytes(K, N) / res["pdl"] / 1e3, 1)}

    # ---- the whole config-1 sweep: bits in {4, 8} x M in {1, 4, 16}, one graph over COPIES
    # copies of the five shapes per point (weights from HBM), GB/s of algorithmic bytes
    sweep = {}
    if world == 1 and not args.skip_extra:
        for bits in (4, 8):
            ws = [(L[0], L[1], L[2], L[3], L[4]) for L in lay] if bits == 4 else \
                 [(K, N) + tuple(rand_gptq(K, N, dev, g, bits=bits)) for _ in range(COPIES) for (K, N) in SHAPES]
            for M in (1, 4, 16):
                xs = {K: torch.randn((M, K), device=dev, generator=g).half() for K, _ in SHAPES}
                ys = {N: torch.empty((M, N), device=dev) for _, N in SHAPES}

                def one_pass():
                    for (K, N, qw, qz, sc) in ws:
                        _gptq_matmul(xs[K], qw, qz, sc, K, N, GS, bits, 1.0, out=ys[N])
                one_pass()
                torch.cuda.synchronize()
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr):
                    one_pass()
                for _ in range(3):
                    gr.replay()
                us = event_time(gr.replay, 20) * 1e3
                nbytes = sum(gemv_bytes(K, N, M=M, bits=bits) for (K, N, _, _, _) in ws)
                sweep["int%d_M%d" % (bits, M)] = {"us_per_pass": round(us, 2),
                                                   "GB/s": round(nbytes / us / 1e3, 1),
                                                   "frac_of_hbm": round(nbytes / us / 1e3 / peaks()[0], 4)}
                del gr, xs, ys
            del ws
        torch.cuda.empty_cache()

    # ---- e2e: public operator path with pinned host buffers, copies inside the timed region.
    # A step uploads its 20 activation rows (packed in one pinned buffer) with one copy, makes
    # the 20 operator calls, and reads back the packed outputs (all ranks' after the all-gather).
    x_off, xo = [], 0
    for L in lay:
        x_off.append(xo)
        xo += L[0]
    x_all = torch.empty((1, xo), device=dev, dtype=torch.float16)
    lay_e2e = []
    for L, o in zip(lay, x_off):
        x_all[:, o:o + L[0]].copy_(L[5])
        lay_e2e.append(L[:5] + (x_all[:, o:o + L[0]], L[6]))
    hx = torch.empty(x_all.shape, dtype=x_all.dtype, pin_memory=True).copy_(x_all.cpu())
    hy = torch.empty((world, n_out) if world > 1 else y_all.shape, dtype=y_all.dtype, pin_memory=True)
    h2d = hx.numel() * hx.element_size()
    d2h = hy.numel() * hy.element_size()

    def e2e_step():
        x_all.copy_(hx, non_blocking=True)
        for L in lay_e2e:
            launch(L)
        if world > 1:
            dist.all_gather_into_tensor(gathered, y_all)
            hy.copy_(gathered, non_blocking=True)
        else:
            hy.copy_(y_all, non_blocking=True)

    for _ in range(3):
        e2e_step()
    e2e_steps = max(1, min(args.steps, 500))
    ems, _, _ = timed(e2e_step, e2e_steps)

    # ---- config 3: prefill dequant-GEMM (tcgen05), desc_act, bf16 x, M = 2048
    gemm = {}
    if not args.skip_gemm and world == 1:
        from webpytorch_b200.qlinear import QuantizedLinear
        _, bf16_peak, _ = peaks()
        for (K, N) in GEMM_SHAPES:
            qw, qz, sc = rand_gptq(K, N, dev, g)
            gidx = (torch.arange(K, device=dev) // GS)[torch.randperm(K, device=dev, generator=g)]
            ql = QuantizedLinear.from_autogptq(qw, qz, sc, None, GS, 4, g_idx=gidx, device=dev)
            for M in GEMM_MS:
                x = torch.randn((M, K), device=dev, generator=g).to(torch.bfloat16)
                yb = torch.empty((M, N), device=dev, dtype=torch.bfloat16)
                for _ in range(3):
                    ql(x, out=yb, out_dtype=torch.bfloat16)
                us = event_time(lambda: ql(x, out=yb, out_dtype=torch.bfloat16), 20) * 1e3
                tflops = 2.0 * M * N * K / (us * 1e-6) / 1e12
                gemm["%dx%d_M%d" % (K, N, M)] = {"us": round(us, 2), "TFLOP/s": round(tflops, 1),
                                                  "frac_of_bf16_peak": round(tflops / bf16_peak, 4)}
                del x, yb
            del ql, qw, qz, sc
        torch.cuda.empty_cache()

    moe_res, q4k_res, moe_ep, dec_res = {}, {}, {}, {}
    if not args.skip_extra:
        hbm0, bf0, _ = peaks()
        if world == 1:
            q4k_res = bench_q4k(dev, g, hbm0)
            moe_res = bench_moe(dev, g, hbm0, bf0)
            dec_res = bench_decode(dev, g, hbm0)
            torch.cuda.empty_cache()
        moe_ep = bench_moe_ep(dev, g, world, timed)

    tot_bytes = step_bytes() * args.steps * world
    value = tot_bytes / (ms / 1e3) / 1e9
    value_pdl = tot_bytes / (ms_pdl / 1e3) / 1e9
    e2e_value = step_bytes() * e2e_steps * world / (ems / 1e3) / 1e9
    hbm, _, src = peaks()
    launches_per_step = len(lay)
    avg_launch_us = ms * 1e3 / (args.steps * launches_per_step)
    achieved = step_bytes() / launches_per_step / (avg_launch_us * 1e3)   # GB/s
    result = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int4 weights, fp16 x, fp32 accumulate/out",
        "data": "synthetic",
        "config": workload_config(world),
        "step": {"gemvs": len(lay), "copies": COPIES, "MB": round(step_bytes() / 1e6, 1), "cuda_graph": True,
                 "launch": "plain graph launches (value_with_pdl: QL_LAUNCH_PDL)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4),
                     "traffic": round(GEMV_TRAFFIC_RATIO * step_bytes() / launches_per_step),
                     "traffic_basis": "ncu dram read+write of one 4096x14336 launch, scaled per launch by "
                                      "algorithmic bytes (bytes per launch, averaged over the sweep)",
                     "peak_source": "%s (MEASURED_PEAKS.json hbm_gbs)" % src if src == "measured" else src,
                     "avg_launch_us": round(avg_launch_us, 3)},
        "value_with_pdl": round(value_pdl, 2),
        "per_shape": per_shape,
        "config1_sweep": {"basis": "one pass = %d GEMVs (%d copies of the 5 shapes, weights from HBM), fp16 x, "
                                   "fp32 out; algorithmic bytes / pass time" % (COPIES * len(SHAPES), COPIES),
                          "points": sweep},
        "gemm": {"workload": "config3: int4 g128 desc_act dequant-GEMM, bf16 x/out, M in %s (act-order gather "
                             "+ fp16 staging + tcgen05 GEMM per call)" % (GEMM_MS,),
                 "bound": "tensor", "peak_TFLOP/s": peaks()[1], "shapes": gemm},
        "q4k": {"workload": "config2: Q4_K K=%d N=%d fp32 x/out, %d rotating copies (%.0f MB)"
                            % (Q4K_K, Q4K_N, Q4K_COPIES, Q4K_COPIES * Q4K_N * Q4K_K / 256 * 144 / 1e6),
                "bound": "hbm", "M": q4k_res},
        "moe": {"workload": "config4: %d experts top-%d, H=%d I=%d, int4 g128, bf16 x, device routing + "
                            "grouped gate|up + act + grouped down + combine per layer, CUDA graph over "
                            "independent layers" % (MOE_E, MOE_TOPK, MOE_H, MOE_I),
                "expert_GB/s basis": "active experts' packed weights+scales+zeros per layer / layer time",
                "T": moe_res},
        "moe_ep": moe_ep,
        "decode": dec_res,
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                "path": "eager calls of the operator boundary (_gptq_matmul via ctypes), one pinned-host "
                        "upload of the step's 20 activation rows and one read-back of its outputs per step"},
        "gpu_launches": args.steps * launches_per_step,
        "clocks": clocks,
    }
    if world == 1 and rank == 0 and args.cpu_seconds > 0:
        result["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
    if rank == 0:
        json_out.write(json.dumps(result) + "\n")
        json_out.flush()
    del graph, graph_pdl
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
