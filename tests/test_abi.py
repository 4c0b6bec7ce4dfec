"""The C-ABI library loads on the host and exports exactly what include/*.h declares (CPU only).

Argument validation happens on the host before any CUDA call, so bad arguments are checked
here without a GPU.
"""
import ctypes
import glob
import os
import re

import pytest

from webpytorch_b200 import _build, _ffi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        names |= set(re.findall(r"QL_API\s+[\w\s\*]+?\b(ql_\w+)\s*\(", src))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    _build.build()
    return _ffi.load()


def test_library_exports_every_declared_symbol(lib):
    names = declared_symbols()
    assert "ql_gptq_matmul" in names and len(names) >= 5
    raw = ctypes.CDLL(_ffi.lib_path())
    for n in names:
        assert hasattr(raw, n), n
    assert set(names) <= set(_ffi.SIGNATURES), set(names) - set(_ffi.SIGNATURES)


def test_version_and_empty_error(lib):
    assert lib.ql_version() >= 100
    assert lib.ql_last_error() is not None


def _matmul_rc(lib, **kw):
    a = dict(x=1, x_dtype=1, ldx=128, x_perm=None, qw=16, qz=16, sc=16, sc_dtype=1, bias=None, out=16,
             out_dtype=0, ldo=64, M=1, K=128, N=64, gs=128, bits=4, zoff=1.0)
    a.update(kw)
    v = ctypes.c_void_p
    return lib.ql_gptq_matmul(v(a["x"]), a["x_dtype"], a["ldx"], v(a["x_perm"]) if a["x_perm"] else None,
                              v(a["qw"]), v(a["qz"]), v(a["sc"]), a["sc_dtype"], a["bias"], v(a["out"]),
                              a["out_dtype"], a["ldo"], a["M"], a["K"], a["N"], a["gs"], a["bits"],
                              a["zoff"], None)


@pytest.mark.parametrize("kw,code", [
    (dict(bits=5), 3), (dict(bits=2), 3), (dict(K=130), 1), (dict(gs=0), 1), (dict(N=60), 1),
    (dict(x_dtype=7), 1), (dict(out_dtype=9), 1), (dict(M=-1), 1), (dict(x=0), 1), (dict(ldx=64), 1),
    (dict(gs=16, K=128), 3), (dict(zoff=0.5), 3), (dict(qw=8), 2), (dict(N=68, ldo=68), 1),
])
def test_matmul_rejects_bad_arguments_on_host(lib, kw, code):
    assert _matmul_rc(lib, **kw) == code
    assert lib.ql_last_error()


def test_matmul_m_zero_is_a_noop(lib):
    assert _matmul_rc(lib, M=0) == 0


def test_other_entry_points_reject_bad_arguments(lib):
    v = ctypes.c_void_p
    assert lib.ql_gptq_dequant(v(16), v(16), v(16), 1, None, v(16), 128, 64, 128, 3, 0.0, None) == 3
    assert lib.ql_gptq_sort_rows(v(16), v(16), v(16), 128, 64, 6, None) == 3
    assert lib.ql_gptq_sort_rows(v(16), v(16), v(16), 127, 64, 4, None) == 1
    assert lib.ql_gptq_sort_rows(v(16), v(16), v(16), 128, 64, 4, None) == 1  # aliasing


def test_q4k_entry_points_reject_bad_arguments(lib):
    v = ctypes.c_void_p
    assert lib.ql_q4k_dequant(v(16), v(16), 4, 100, None) == 1                 # K % 256
    assert lib.ql_q4k_matmul(v(16), 5, 256, v(16), None, v(16), 0, 4, 1, 256, 4, None) == 1    # dtype
    assert lib.ql_q4k_matmul(v(16), 0, 256, v(8), None, v(16), 0, 4, 1, 256, 4, None) == 2     # raw align
    assert lib.ql_q4k_matmul(v(16), 0, 256, v(16), None, v(16), 0, 4, 0, 256, 4, None) == 0    # M == 0
    assert lib.ql_q4k_matmul(v(16), 0, 100, v(16), None, v(16), 0, 4, 1, 256, 4, None) == 1    # ldx < K


def test_launch_flags_roundtrip(lib):
    old = lib.ql_set_launch_flags(1)
    assert lib.ql_set_launch_flags(old) == 1


def test_moe_entry_points_reject_bad_arguments(lib):
    v = ctypes.c_void_p
    p = [v(16)] * 12
    # ql_moe_route: E above the device scan's limit, top_k above E, top_k above 16
    for T, E, k in [(4, 1025, 2), (4, 8, 9), (4, 64, 17), (-1, 8, 2)]:
        assert lib.ql_moe_route(p[0], T, E, k, 1, 128, *p[:9], 4, *p[:2], None) == 1
    assert lib.ql_moe_route(p[0], 4, 8, 2, 1, 128, *p[:9], 4, None, p[0], None) == 1   # null buffer
    assert lib.ql_moe_route(None, 4, 8, 2, 1, 128, *p[:9], 4, *p[:2], None) == 1

    def gm(**kw):
        a = dict(x=16, x_dtype=0, ldx=256, P=8, qw=16, sc=16, sc_dtype=1, E=4, K=256, N=64, gs=128, bits=4,
                 zoff=1.0, ldo=64)
        a.update(kw)
        return lib.ql_moe_grouped_matmul(v(a["x"]), a["x_dtype"], a["ldx"], None, a["P"], v(a["qw"]), v(16),
                                         v(a["sc"]), a["sc_dtype"], a["E"], v(16), v(16), v(16), None, None, 0,
                                         128, 4, v(16), 0, a["ldo"], a["K"], a["N"], a["gs"], a["bits"],
                                         a["zoff"], None, 0, None)
    for kw, code in [(dict(bits=3), 3), (dict(N=60, ldo=60), 1), (dict(K=200), 1), (dict(E=0), 1),
                     (dict(x_dtype=5), 1), (dict(zoff=0.5), 3), (dict(qw=8), 2), (dict(ldx=100), 1),
                     (dict(P=-1), 1)]:
        assert gm(**kw) == code, kw
    assert gm(P=0) == 0
    assert lib.ql_moe_grouped_workspace(0, 8, 256, 128) == 0
    assert lib.ql_moe_grouped_workspace(4096, 8, 256, 128) >= 4096 * 256 * 2   # tensor-core path stages x
    assert lib.ql_moe_act(v(16), 4, 0, v(16), 0, None) == 1
    assert lib.ql_moe_act(v(16), 0, 8, v(16), 0, None) == 0
    assert lib.ql_moe_combine(v(16), v(16), v(16), 2, 2, 64, None, 0, None, 0, v(16), 0, 32, None) == 1
    assert lib.ql_moe_combine(v(16), v(16), v(16), 2, 2, 64, None, 0, v(16), 1, v(16), 0, 64, None) == 1
