"""GGUF Q4_K on the GPU against the reference's dequantiser outputs (golden) and the oracle."""
import numpy as np
import pytest
import torch

from conftest import golden, max_rel_err, same_bits_or_both_nan
from oracle import q4k as oq
from webpytorch_b200 import synth
from webpytorch_b200.ggml import GGMLLinear, ggml_matmul, q4k_dequant

pytestmark = pytest.mark.gpu
TOL = 2e-3
DEV = "cuda"


def _raw(a):
    return torch.from_numpy(np.ascontiguousarray(a).reshape(-1).view(np.uint8)).to(DEV)


@pytest.mark.parametrize("name", ["q4k_randombytes.npz", "q4k_synth.npz", "q4k_rawbytes_nonfinite.npz"])
def test_dequant_bitexact_vs_reference(name):
    d = golden(name)
    N, K = int(d["N"]), int(d["K"])
    W = q4k_dequant(_raw(d["raw"]), K, N).cpu().numpy()
    assert same_bits_or_both_nan(W, d["W"])


def test_matmul_vs_reference_randombytes():
    d = golden("q4k_randombytes.npz")
    lin = GGMLLinear(d["raw"].tobytes(), "Q4_K", int(d["K"]), int(d["N"]))
    y = lin(torch.from_numpy(d["x"]).to(DEV)).cpu().numpy()
    assert max_rel_err(y, d["y"]) < TOL


@pytest.mark.parametrize("M", [1, 8, 13])
@pytest.mark.parametrize("xdt", [torch.float32, torch.float16, torch.bfloat16])
def test_matmul_vs_reference_synth(M, xdt):
    d = golden("q4k_synth.npz")
    N, K = int(d["N"]), int(d["K"])
    lin = GGMLLinear(d["raw"], "Q4_K", K, N)
    x = torch.from_numpy(d["x_%d" % M]).to(DEV).to(xdt)
    y = lin(x).cpu().numpy()
    ref = d["y_%d" % M] if xdt == torch.float32 else oq.matmul(x.float().cpu().numpy(), d["raw"].tobytes(), K, N)
    assert max_rel_err(y, ref) < TOL


@pytest.mark.parametrize("M", [1, 3, 8, 16, 17, 64])
def test_config2_full_size(M):
    """Config 2 shape (K=4096, N=14336) against the exact dequant (bit-exact above) in fp64."""
    N, K = 14336, 4096
    raw = synth.q4k_weights(N, K, seed=M)
    rd = _raw(raw)
    W = q4k_dequant(rd, K, N).double()
    x = torch.randn((M, K), device=DEV, generator=torch.Generator(device=DEV).manual_seed(M))
    y = ggml_matmul(x, rd, "Q4_K", K, N)
    ref = x.double() @ W.T
    assert max_rel_err(y.cpu().numpy(), ref.cpu().numpy()) < TOL
    # a slab of the exact dequant against the oracle at full size
    ref_w = oq.dequant(raw[:64].tobytes(), 64 * K).reshape(64, K)
    assert np.array_equal(W[:64].float().cpu().numpy().view(np.uint32), ref_w.view(np.uint32))


@pytest.mark.parametrize("M,N,K", [(16, 400, 2816), (64, 384, 1024), (128, 2048, 768), (300, 528, 4096),
                                   (40, 37, 768)])
@pytest.mark.parametrize("xdt", [torch.float32, torch.bfloat16])
def test_tensor_core_path_vs_exact_dequant(M, N, K, xdt):
    """M >= 16 takes the tcgen05 GEMM (super-blocks dequantised into TMEM; N % 16 != 0 stays on the
    decode kernels): against the exact dequant in fp64 with a bias, ragged token and row tiles."""
    rng = np.random.default_rng(M + N)
    raw = synth.q4k_weights(N, K, rng=rng)
    bias = rng.standard_normal(N).astype(np.float32)
    lin = GGMLLinear(raw.tobytes(), "Q4_K", K, N, bias=bias)
    x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(DEV).to(xdt)
    y = lin(x)
    W = q4k_dequant(_raw(raw), K, N).double()
    ref = x.double() @ W.T + torch.from_numpy(bias).to(DEV).double()
    assert max_rel_err(y.cpu().numpy(), ref.cpu().numpy()) < TOL


@pytest.mark.parametrize("M", [3, 8, 16, 64])
def test_workspace_entry_matches(M):
    """ql_q4k_matmul_ws with a workspace of ql_q4k_matmul_workspace(M, K) bytes gives the same
    result as ql_q4k_matmul (which takes its staging from the stream-ordered allocator)."""
    from webpytorch_b200 import _ffi
    N, K = 256, 1024
    raw = _raw(synth.q4k_weights(N, K, seed=M))
    x = torch.randn((M, K), device=DEV, generator=torch.Generator(device=DEV).manual_seed(M))
    ref = ggml_matmul(x, raw, "Q4_K", K, N)
    nbytes = int(_ffi.fn("ql_q4k_matmul_workspace")(M, K))
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=DEV)
    out = torch.empty((M, N), device=DEV)
    _ffi.call("ql_q4k_matmul_ws", x.data_ptr(), _ffi.dtype_code(x.dtype), x.stride(0), raw.data_ptr(), None,
              out.data_ptr(), _ffi.dtype_code(out.dtype), out.stride(0), M, K, N, ws.data_ptr(), nbytes,
              _ffi.stream_ptr())
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


@pytest.mark.parametrize("K", [768, 256, 2816])
def test_bias_ragged_rows_and_host_io(K):
    rng = np.random.default_rng(3)
    N = 37                             # N not a multiple of the 16-row warp tile; K-split ranks get
                                       # unequal block counts
    raw = synth.q4k_weights(N, K, rng=rng)
    bias = rng.standard_normal(N).astype(np.float32)
    lin = GGMLLinear(raw.tobytes(), "Q4_K", K, N, bias=bias)
    x = rng.standard_normal((2, 3, K)).astype(np.float32)
    y = lin(torch.from_numpy(x))
    assert y.device.type == "cpu" and tuple(y.shape) == (2, 3, N)
    ref = oq.matmul(x.reshape(-1, K), raw.tobytes(), K, N, bias).reshape(2, 3, N)
    assert max_rel_err(y.numpy(), ref) < TOL


def test_unsupported_type_raises():
    with pytest.raises(NotImplementedError):
        GGMLLinear(b"\x00" * 84, "Q2_K", 256, 1)
