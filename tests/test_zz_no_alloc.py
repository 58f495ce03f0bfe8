"""jc_gemm_noalloc: the split-K GEMM for callers that cannot allocate device memory (its scratch is a
fixed array inside the library), called through the C ABI and checked against jc_gemm, which takes
its scratch from the caller. Two calls in a row, because every call shares the fixed scratch and
the second must not see the first's leftovers. Kept in a file of its own that pytest collects
last."""
import ctypes
import importlib

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


@pytest.fixture(scope="module")
def noalloc():
    jc = importlib.import_module("julia-cuda_b200")
    lib = ctypes.CDLL(jc.LIB_PATH)
    fn = lib.jc_gemm_noalloc
    P, u32, i32, f32 = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int, ctypes.c_float
    fn.argtypes = [u32, i32, i32, P, P, P, P, P, P, P, P, u32, u32, u32, u32, f32, P, P, P]
    fn.restype = i32
    lib.jc_last_error.restype = ctypes.c_char_p
    return jc, lib, fn


@pytest.mark.parametrize("epi_name,n,k,splits", [("resstats", 768, 1152, 4),
                                                 ("lngeglu", 2304, 768, 3),
                                                 ("lnbias", 768, 768, 2)])
def test_noalloc_matches_jc_gemm_twice(noalloc, epi_name, n, k, splits):
    jc, lib, fn = noalloc
    epi = jc.EPILOGUES[epi_name]
    m = 293
    g = torch.Generator(device="cuda").manual_seed(n + k)
    a = torch.randn(m, k, device="cuda", generator=g).half()
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.05).half()
    n_out = n // 2 if epi & jc.EPI_GEGLU else n
    res0 = torch.randn(m, n_out, device="cuda", generator=g).half()
    st = (torch.rand(2 * m, device="cuda", generator=g) + 1.0).contiguous()
    st[1::2] += 800.0
    cs = torch.randn(n, device="cuda", generator=g)
    bias = torch.randn(n, device="cuda", generator=g)
    stream = torch.cuda.current_stream().cuda_stream

    # the existing entry point, scratch from the caller
    want = res0.clone()
    want_st = torch.zeros(2 * m, device="cuda")
    jc.gemm(epi, a, w, want, res=want if epi & jc.EPI_RES else None, stats_in=st, colsum=cs,
            stats_out=want_st, bias=bias, bn=64, splits=splits)
    torch.cuda.synchronize()

    for call in range(2):
        got = res0.clone()
        got_st = torch.zeros(2 * m, device="cuda")
        rc = fn(epi, 64, splits, ptr(a), ptr(w), ptr(got), ptr(got) if epi & jc.EPI_RES else None,
                ptr(st), ptr(cs), ptr(got_st), None, 0, m, n, k, 1e-5, None, ptr(bias), stream)
        assert rc == 0, lib.jc_last_error()
        torch.cuda.synchronize()
        g32, w32 = got.float(), want.float()
        err = float((g32 - w32).norm() / w32.norm())
        assert err < 1e-3, f"call {call}: rel err {err:.2e}"
        if epi & jc.EPI_STATS:
            assert torch.allclose(got_st, want_st, rtol=1e-4, atol=1e-3)


def test_noalloc_rejects_scratch_overflow(noalloc):
    jc, lib, fn = noalloc
    m, n, k = 1024, 2304, 2048
    a = torch.zeros(m, k, device="cuda").half()
    w = torch.zeros(n, k, device="cuda").half()
    c = torch.zeros(m, n, device="cuda").half()
    rc = fn(0, 64, 8, ptr(a), ptr(w), ptr(c), None, None, None, None, None, 0, m, n, k, 1e-5, None,
            None, torch.cuda.current_stream().cuda_stream)
    assert rc == -1 and b"scratch" in lib.jc_last_error()
