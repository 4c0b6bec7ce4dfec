"""MoE block on the GPU against the oracle (a restatement of lm_engine.moe_mlp) and the reference's
own outputs (tests/golden/moe_*.npz, made by importing the reference)."""
import numpy as np
import pytest
import torch

from conftest import golden, golden_files, max_rel_err
from oracle import gptq as og
from oracle import moe as om
from webpytorch_b200 import moe, synth
from webpytorch_b200.qlinear import QuantizedLinear

pytestmark = pytest.mark.gpu
TOL = 2e-3
DEV = "cuda"


def _ql(w, gs, bits):
    return QuantizedLinear.from_autogptq(w["qweight"], w["qzeros"], w["scales"], None, gs, bits, device=DEV)


def _oracle_lin(w, K, N, gs, bits):
    return lambda x: og.quantized_linear(x, w["qweight"], w["qzeros"], w["scales"], None, K, N, K, N, gs, bits, 1.0)


def _check_routing(r, logits, top_k, norm):
    T, E = logits.shape
    idx = r.topk_idx.cpu().numpy()
    w = r.topk_w.cpu().numpy()
    ref_idx, ref_w = om.route(logits, top_k, norm)
    for t in range(T):
        o, ro = np.argsort(idx[t]), np.argsort(ref_idx[t])
        assert np.array_equal(idx[t][o], ref_idx[t][ro]), t
        np.testing.assert_allclose(w[t][o], ref_w[t][ro], rtol=1e-6, atol=1e-7)
    counts = np.bincount(idx.ravel(), minlength=E)
    assert np.array_equal(r.counts.cpu().numpy(), counts)
    offs = np.concatenate([[0], np.cumsum(counts)])
    assert np.array_equal(r.offsets.cpu().numpy(), offs)
    act = np.nonzero(counts)[0]
    assert int(r.n_active.item()) == len(act)
    assert np.array_equal(r.active.cpu().numpy()[:len(act)], act)
    row_token = r.row_token.cpu().numpy()[:T * top_k]
    pair_row = r.pair_row.cpu().numpy()
    assert sorted(pair_row.ravel().tolist()) == list(range(T * top_k))
    for t in range(T):
        for j in range(top_k):
            p = pair_row[t, j]
            e = idx[t, j]
            assert row_token[p] == t and offs[e] <= p < offs[e + 1]
    tiles = [(e, s) for e in act for s in range(0, counts[e], moe.TILE_ROWS)]
    assert int(r.n_tiles.item()) == len(tiles)
    assert np.array_equal(r.tiles.cpu().numpy()[:2 * len(tiles)].reshape(-1, 2), np.array(tiles).reshape(-1, 2))


@pytest.mark.parametrize("T,E,k,norm", [(1, 8, 2, True), (37, 64, 8, True), (300, 128, 8, False),
                                        (5, 1000, 16, True), (64, 16, 1, True),
                                        (700, 64, 8, True), (2048, 128, 8, True)])   # multi-kernel route
def test_route_matches_oracle(T, E, k, norm):
    rng = np.random.default_rng(T * 7 + E)
    logits = rng.standard_normal((T, E)).astype(np.float32)
    r = moe.route(torch.from_numpy(logits).to(DEV), k, norm)
    torch.cuda.synchronize()
    _check_routing(r, logits, k, norm)


def test_route_ties_pick_lower_expert():
    logits = np.zeros((3, 8), np.float32)
    logits[1, 5] = 1.0
    r = moe.route(torch.from_numpy(logits).to(DEV), 2)
    idx = np.sort(r.topk_idx.cpu().numpy(), 1)
    assert idx[0].tolist() == [0, 1] and idx[1].tolist() == [0, 5] and idx[2].tolist() == [0, 1]


def _block_from_fixture(d):
    E, top_k, gs, bits = (int(d[k]) for k in ("E", "top_k", "gs", "bits"))

    def q(pre, k):
        return _ql({f: d["%s_%s_%s" % (pre, k, f)] for f in ("qweight", "qzeros", "scales")}, gs, bits)
    experts = [{k: q("e%d" % e, k) for k in ("gate", "up", "down")} for e in range(E)]
    logits = torch.from_numpy(d["logits"]).to(DEV)
    shared = shared_gate = None
    if "SI" in d:
        shared = {k: q("shared", k) for k in ("gate", "up", "down")}
        gw = torch.from_numpy(d["shared_gate_w"]).to(DEV)
        shared_gate = (lambda x: x @ gw)
    norm = bool(int(d["norm_topk_prob"])) if "norm_topk_prob" in d else True
    return moe.MoEBlock(lambda x: logits, experts, top_k, norm, shared, shared_gate)


@pytest.mark.parametrize("name", golden_files("moe_"))
def test_moe_block_vs_reference_fixture(name):
    d = golden(name)
    blk = _block_from_fixture(d)
    y = blk(torch.from_numpy(d["x"]).to(DEV))
    torch.cuda.synchronize()
    assert max_rel_err(y.cpu().numpy(), d["y"]) < TOL


def test_moe_function_level_dropin():
    """moe_mlp(lm, lay, x) takes the reference's own layer dict (QuantizedLinear experts)."""
    d = golden("moe_E8_k2_T5.npz")
    E, top_k, gs, bits = (int(d[k]) for k in ("E", "top_k", "gs", "bits"))
    logits = torch.from_numpy(d["logits"]).to(DEV)
    experts = [{k: _ql({f: d["e%d_%s_%s" % (e, k, f)] for f in ("qweight", "qzeros", "scales")}, gs, bits)
                for k in ("gate", "up", "down")} for e in range(E)]
    lay = {"moe": {"gate": (lambda x: logits), "experts": experts, "top_k": top_k, "norm_topk_prob": True,
                   "shared": None}}
    x = torch.from_numpy(d["x"]).to(DEV)
    y = moe.moe_mlp(None, lay, x)
    assert max_rel_err(y.cpu().numpy(), d["y"]) < TOL
    assert torch.equal(moe.moe_mlp(None, lay, x), y)     # the cached block is reused


def _synthetic_case(E, H, I, T, k, bits, seed, skew=0.0, shared=False):
    rng = np.random.default_rng(seed)
    exps = synth.moe_experts(E, H, I, bits=bits, gs=128, rng=rng)
    logits = rng.standard_normal((T, E)).astype(np.float32)
    if skew:
        logits[:, 3] += skew                        # one expert takes (nearly) every token
    x = rng.standard_normal((T, H)).astype(np.float32)
    sh = synth.moe_experts(1, H, I, bits=bits, gs=128, rng=rng)[0] if shared else None
    return exps, logits, x, sh


@pytest.mark.parametrize("E,H,I,T,k,bits,skew", [
    (8, 512, 256, 300, 2, 4, 0.0),     # ~75 rows per expert: tensor-core grouped GEMM
    (8, 512, 256, 260, 2, 8, 0.0),
    (16, 256, 128, 200, 1, 4, 30.0),   # every token on expert 3: GEMV walks 13 chunks of one expert
    (64, 1024, 512, 4, 8, 4, 0.0),     # decode: grouped GEMV over the active experts
    (64, 1024, 512, 16, 8, 8, 0.0),
])
def test_moe_block_vs_oracle(E, H, I, T, k, bits, skew):
    exps, logits, x, _ = _synthetic_case(E, H, I, T, k, bits, seed=E + T, skew=skew)
    experts = [{p: _ql(e[p], 128, bits) for p in ("gate", "up", "down")} for e in exps]
    lg = torch.from_numpy(logits).to(DEV)
    blk = moe.MoEBlock(lambda t: lg, experts, k)
    y = blk(torch.from_numpy(x).to(DEV)).cpu().numpy()
    ref_experts = [(_oracle_lin(e["gate"], H, I, 128, bits), _oracle_lin(e["up"], H, I, 128, bits),
                    _oracle_lin(e["down"], I, H, 128, bits)) for e in exps]
    ref = om.moe_mlp(x, logits, ref_experts, k)
    assert max_rel_err(y, ref) < TOL


def test_moe_shared_expert_prefill_vs_oracle():
    E, H, I, T, k = 8, 256, 256, 192, 2
    exps, logits, x, sh = _synthetic_case(E, H, I, T, k, 4, seed=5, shared=True)
    gw = (np.random.default_rng(6).standard_normal((H, 1)) * 0.05).astype(np.float32)
    experts = [{p: _ql(e[p], 128, 4) for p in ("gate", "up", "down")} for e in exps]
    lg = torch.from_numpy(logits).to(DEV)
    gwd = torch.from_numpy(gw).to(DEV)
    blk = moe.MoEBlock(lambda t: lg, experts, k, True, {p: _ql(sh[p], 128, 4) for p in ("gate", "up", "down")},
                       lambda t: t @ gwd)
    y = blk(torch.from_numpy(x).to(DEV)).cpu().numpy()
    lin = _oracle_lin
    ref = om.moe_mlp(x, logits, [(lin(e["gate"], H, I, 128, 4), lin(e["up"], H, I, 128, 4),
                                  lin(e["down"], I, H, 128, 4)) for e in exps], k, True,
                     (lin(sh["gate"], H, I, 128, 4), lin(sh["up"], H, I, 128, 4), lin(sh["down"], I, H, 128, 4)),
                     lambda t: t @ gw)
    assert max_rel_err(y, ref) < TOL


@pytest.mark.parametrize("T", [3, 333])
def test_moe_block_is_deterministic(T):
    exps, logits, x, _ = _synthetic_case(16, 512, 256, T, 4, 4, seed=T)
    experts = [{p: _ql(e[p], 128, 4) for p in ("gate", "up", "down")} for e in exps]
    lg = torch.from_numpy(logits).to(DEV)
    blk = moe.MoEBlock(lambda t: lg, experts, 4)
    xd = torch.from_numpy(x).to(DEV)
    a = blk(xd)
    b = blk(xd)
    assert torch.equal(a, b)


def test_moe_block_empty_batch():
    exps, logits, x, _ = _synthetic_case(4, 256, 128, 1, 2, 4, seed=1)
    experts = [{p: _ql(e[p], 128, 4) for p in ("gate", "up", "down")} for e in exps]
    blk = moe.MoEBlock(lambda t: torch.zeros((0, 4), device=DEV), experts, 2)
    y = blk(torch.zeros((0, 256), device=DEV))
    assert y.shape == (0, 256)


@pytest.mark.parametrize("H,shared,out_dtype", [(2048, False, torch.float32), (2048, True, torch.bfloat16),
                                                 (2050, True, torch.float32), (12, False, torch.float16)])
def test_combine_matches_ordered_sum(H, shared, out_dtype):
    """ql_moe_combine (16-byte column path for H % 4 == 0, element path otherwise) against the
    ordered fp32 sum sum_j w[t, j] * z[pair_row[t, j]] (+ sigmoid(g_t) * shared[t])."""
    from webpytorch_b200 import _ffi
    T, k = 37, 8
    rng = np.random.default_rng(H)
    z = rng.standard_normal((T * k, H)).astype(np.float32)
    pair = rng.permutation(T * k).astype(np.int32).reshape(T, k)
    w = rng.random((T, k)).astype(np.float32)
    sh = rng.standard_normal((T, H)).astype(np.float32) if shared else None
    gl = rng.standard_normal((T, 1)).astype(np.float32) if shared else None
    out = torch.empty((T, H), dtype=out_dtype, device=DEV)
    zd, pd, wd = (torch.from_numpy(a).to(DEV) for a in (z, pair, w))
    shd = torch.from_numpy(sh).to(DEV) if shared else None
    gld = torch.from_numpy(gl).to(DEV) if shared else None
    _ffi.call("ql_moe_combine", zd.data_ptr(), pd.data_ptr(), wd.data_ptr(), T, k, H, _ffi.ptr(shd),
              H if shared else 0, _ffi.ptr(gld), 1 if shared else 0, out.data_ptr(), _ffi.dtype_code(out_dtype),
              H, _ffi.stream_ptr())
    ref = np.zeros((T, H), np.float64)
    for j in range(k):
        ref += w[:, j:j + 1].astype(np.float64) * z[pair[:, j]]
    if shared:
        ref += sh / (1.0 + np.exp(-gl.astype(np.float64)))
    tol = 1e-5 if out_dtype == torch.float32 else 1e-2
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, rtol=tol, atol=tol)


def test_moe_step_replays_in_a_cuda_graph():
    exps, logits, x, _ = _synthetic_case(32, 512, 256, 4, 4, 4, seed=9)
    experts = [{p: _ql(e[p], 128, 4) for p in ("gate", "up", "down")} for e in exps]
    lg = torch.from_numpy(logits).to(DEV)
    blk = moe.MoEBlock(lambda t: lg, experts, 4)
    xd = torch.from_numpy(x).to(DEV)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ref = blk(xd)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            out = blk(xd)
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


@pytest.mark.parametrize("E,K,N,T,k,bits,gs", [
    (16, 256, 256, 12, 8, 4, 64),     # cluster split over 2 stages, 16-row chunks
    (16, 128, 256, 12, 8, 4, 64),     # one stage, no split
    (8, 256, 256, 5, 2, 4, 64),
    (8, 1024, 512, 3, 2, 4, 128),
    (8, 1024, 512, 12, 4, 8, 128),
    (4, 2048, 1536, 40, 2, 4, 128),   # more rows than a chunk: several chunks per expert
])
@pytest.mark.parametrize("xdtype,gather", [(torch.float16, True), (torch.float32, True), (torch.float32, False)])
@pytest.mark.parametrize("table", ["chosen", "128", "64", "32"])
def test_grouped_matmul_vs_dense_per_expert(E, K, N, T, k, bits, gs, xdtype, gather, table):
    """Every expert's sorted rows of ql_moe_grouped_matmul equal the dense operator on its weights
    (rows gathered through row_token, or read in sorted order directly), with the tile table the
    call asks for (tensor-core GEMM or decode GEMV) and with 128-, 64- and 32-row tiles (the
    tensor-core GEMM's tile heights when the call takes it, else the other paths)."""
    exps = synth.moe_experts(E, K, N, bits=bits, gs=gs, seed=E * T + K)
    experts = [{"gate": _ql(e["gate"], gs, bits), "up": _ql(e["up"], gs, bits), "down": _ql(e["down"], gs, bits)}
               for e in exps]
    w = moe.StackedExperts(experts, ("gate",), DEV)
    rng = np.random.default_rng(T)
    logits = torch.from_numpy(rng.standard_normal((T, E)).astype(np.float32)).to(DEV)
    x = torch.from_numpy(rng.standard_normal((T, K)).astype(np.float32)).to(DEV).to(xdtype)
    tr = moe.tile_rows_for(T * k, E, K, gs, T) if table == "chosen" else int(table)
    r = moe.route(logits, k, True, tr)
    rows = r.row_token[:r.P].long()
    if gather:
        y = moe.grouped_matmul(x, r.row_token, r, w)
    else:
        xs = x[rows].contiguous()          # rows already in sorted order
        y = moe.grouped_matmul(xs, None, r, w)
    torch.cuda.synchronize()
    offs = r.offsets.cpu().numpy()
    rows = rows.cpu().numpy()
    for e in range(E):
        if offs[e + 1] == offs[e]:
            continue
        ref = experts[e]["gate"](x[torch.from_numpy(rows[offs[e]:offs[e + 1]]).long().to(DEV)])
        got = y[offs[e]:offs[e + 1]]
        assert max_rel_err(got.cpu().numpy(), ref.cpu().numpy()) < TOL, (e, offs[e + 1] - offs[e])


@pytest.mark.parametrize("E,K,N,T,k,table,ydt", [
    (16, 768, 256, 300, 8, "chosen", torch.float32),   # tensor-core GEMM, 16-byte staging loads
    (16, 768, 256, 300, 8, "64", torch.float32),
    (16, 768, 256, 300, 8, "32", torch.float16),       # scalar staging loads
    (8, 256, 128, 5, 2, "chosen", torch.float32),      # decode GEMV tiles
    (2, 24704, 64, 40, 1, "128", torch.float32),       # rows beyond the shared-memory staging
])
def test_down_swiglu_equals_act_then_down(E, K, N, T, k, table, ydt):
    """ql_moe_grouped_matmul_swiglu (SwiGLU formed while staging) is bit-identical to ql_moe_act
    into fp32 followed by ql_moe_grouped_matmul, on every tile height and staging path."""
    g = torch.Generator(device=DEV).manual_seed(K + T)
    qw = torch.randint(-2 ** 31, 2 ** 31 - 1, (E, K // 8, N), dtype=torch.int32, device=DEV, generator=g)
    qz = torch.randint(-2 ** 31, 2 ** 31 - 1, (E, K // 128, N // 8), dtype=torch.int32, device=DEV, generator=g)
    sc = (torch.rand((E, K // 128, N), device=DEV, generator=g) * 0.018 + 0.002).half()
    dn = moe.StackedExperts.from_packed(qw, qz, sc, 128, 4)
    logits = torch.randn((T, E), device=DEV, generator=g)
    tr = moe.tile_rows_for(T * k, E, K, 128, T) if table == "chosen" else int(table)
    r = moe.route(logits, k, True, tr)
    y = (torch.randn((r.P, 2 * K), device=DEV, generator=g) * 3).to(ydt)
    got = moe.down_swiglu(y, r, dn)
    ref = moe.grouped_matmul(moe.act(y.float(), K), None, r, dn)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)


@pytest.fixture(scope="module")
def config4_experts():
    """BASELINE config 4 experts: 128 experts, gate|up [2048 -> 2 x 768] and down [768 -> 2048],
    int4 group 128, uniform packed words, fp16 scales U[0.002, 0.02] (generated on the device)."""
    E, H, I = 128, 2048, 768
    g = torch.Generator(device=DEV).manual_seed(44)

    def pack(K, N):
        qw = torch.randint(-2 ** 31, 2 ** 31 - 1, (E, K // 8, N), dtype=torch.int32, device=DEV, generator=g)
        qz = torch.randint(-2 ** 31, 2 ** 31 - 1, (E, K // 128, N // 8), dtype=torch.int32, device=DEV, generator=g)
        sc = (torch.rand((E, K // 128, N), device=DEV, generator=g) * 0.018 + 0.002).half()
        return qw, qz, sc
    gu, dn = pack(H, 2 * I), pack(I, H)
    return E, H, I, gu, dn


@pytest.mark.parametrize("T", [1, 32, 256, 2048])
def test_config4_block_full_size_vs_oracle(config4_experts, T):
    """The config-4 block at full size (128 experts, top-8, H 2048, I 768, bf16 x) against
    oracle/moe.py's moe_mlp (the restatement of webtorch/lm_engine.py:294-329, router replaced by
    the given logits). The oracle's expert linears run in float64 on the exact fp32 dequantised
    weights (ql_gptq_dequant, bit-identical to the reference's unpack: tests above)."""
    from webpytorch_b200.qlinear import gptq_dequant
    E, H, I, gu, dn = config4_experts
    k = 8
    g = torch.Generator(device=DEV).manual_seed(T)
    logits = torch.randn((T, E), device=DEV, generator=g)
    x = torch.randn((T, H), device=DEV, generator=g).to(torch.bfloat16)
    blk = moe.MoEBlock.from_stacked(lambda t: logits, moe.StackedExperts.from_packed(*gu, 128, 4),
                                    moe.StackedExperts.from_packed(*dn, 128, 4), k)
    y = blk(x).cpu().numpy()

    cache = {}

    def weights(e):
        if e not in cache:
            wgu = gptq_dequant(gu[0][e], gu[1][e], gu[2][e], H, 2 * I, 128, 4, 1.0).double()
            wdn = gptq_dequant(dn[0][e], dn[1][e], dn[2][e], I, H, 128, 4, 1.0).double()
            cache[e] = (wgu, wdn)
        return cache[e]

    def lin(e, part):
        def f(a):
            wgu, wdn = weights(e)
            w = wgu[:, :I] if part == 0 else wgu[:, I:] if part == 1 else wdn
            return (torch.from_numpy(np.ascontiguousarray(a, np.float64)).to(DEV) @ w).cpu().numpy()
        return f
    experts = [(lin(e, 0), lin(e, 1), lin(e, 2)) for e in range(E)]
    ref = om.moe_mlp(x.float().cpu().numpy(), logits.cpu().numpy(), experts, k)
    assert max_rel_err(y, ref) < TOL, max_rel_err(y, ref)
