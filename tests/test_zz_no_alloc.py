"""jc_gemm_noalloc: the fused-epilogue GEMM for callers that cannot allocate device memory, whose
split-K scratch is a fixed array inside the library. Called through the C ABI and checked against
the oracle's emulation of the same f16/f32 arithmetic (oracle/oracle.c, the reference's
emulate_gemm, src/check.rs:64-123) with the kernel tests' bars, and against jc_gemm, on two calls
in a row: every call shares the fixed scratch, and the second must not see the first's
leftovers. The cases cover the LayerNorm + RoPE epilogue with the RoPE table passed, GeGLU and
residual + statistics, through workspace split-K (the path that uses the fixed scratch), the
automatic choice (splits 0) and the cluster split (splits -2, no scratch). Kept in a file of its
own that pytest collects last."""
import ctypes
import importlib

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def u16(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda().view(torch.float16)


def f32(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def host_u16(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def elem_err(got, want):
    g = np.asarray(got, np.float64)
    w = np.asarray(want, np.float64)
    floor = 0.1 * max(float(np.sqrt(np.mean(w * w))), 1e-30)
    return float(np.max(np.abs(g - w) / np.maximum(np.abs(w), floor)))


@pytest.fixture(scope="module")
def noalloc():
    jc = importlib.import_module("julia-cuda_b200")
    from oracle import oracle as O
    lib = ctypes.CDLL(jc.LIB_PATH)
    fn = lib.jc_gemm_noalloc
    P, u32, i32, fl = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int, ctypes.c_float
    fn.argtypes = [u32, i32, i32, P, P, P, P, P, P, P, P, u32, u32, u32, u32, fl, P, P, P]
    fn.restype = i32
    lib.jc_last_error.restype = ctypes.c_char_p
    return jc, O, lib, fn


CASES = [  # epilogue, n, k, splits
    ("lnrope", 2304, 768, 3),
    ("lnrope", 2304, 768, 0),
    ("lngeglu", 2304, 768, 4),
    ("lngeglu", 2304, 768, -2),
    ("resstats", 768, 1152, 4),
    ("resstats", 768, 768, 0),
    ("resstats", 768, 1152, -2),
]


@pytest.mark.parametrize("epi_name,n,k,splits", CASES)
def test_noalloc_matches_oracle_twice(noalloc, epi_name, n, k, splits):
    jc, O, lib, fn = noalloc
    epi = jc.EPILOGUES[epi_name]
    m = 293
    seed = n + k + 7 * (splits + 3)
    a = O.f16(O.normal((m, k), seed + 1))
    w = O.f16(O.normal((n, k), seed + 2, std=0.05))
    stats_in = O.row_stats(a)
    colsum = O.f32(w).astype(np.float64).sum(1).astype(np.float32)
    rope = O.rope_table(160000.0, m)
    n_out = n // 2 if epi & jc.EPI_GEGLU else n
    res = O.f16(O.normal((m, n_out), seed + 4))
    want, want_stats = O.emu_gemm(epi, a, w, m, n, k, c16=res if epi & jc.EPI_RES else None,
                                  stats_in=stats_in, colsum=colsum, eps=1e-5, rope=rope)
    w_dev, cs_dev = w, colsum
    if epi & jc.EPI_GEGLU:
        w_dev = jc.prep_interleave_geglu(w)
        cs_dev = jc.prep_interleave_geglu(colsum)
    a_d, w_d, st_d, cs_d = u16(a), u16(w_dev), f32(stats_in), f32(cs_dev)
    rope_d = f32(jc.prep_rope_gemm(rope, m)) if epi & jc.EPI_ROPE else None
    stream = torch.cuda.current_stream().cuda_stream

    # the existing entry point, its scratch from the caller
    ref = u16(res) if epi & jc.EPI_RES else torch.zeros(m, n_out, dtype=torch.float16, device="cuda")
    ref_st = torch.zeros(2 * m, device="cuda")
    bn = 64 if splits < 0 else 0  # a split-K cluster needs 64-column tiles or wider
    jc.gemm(epi, a_d, w_d, ref, res=ref if epi & jc.EPI_RES else None, stats_in=st_d,
            colsum=cs_d, stats_out=ref_st, rope=rope_d, bn=bn, splits=splits)
    torch.cuda.synchronize()
    ref_h = host_u16(ref)

    for call in range(2):
        got = u16(res) if epi & jc.EPI_RES else torch.full((m, n_out), float("nan"),
                                                          dtype=torch.float16, device="cuda")
        got_st = torch.zeros(2 * m, device="cuda")
        rc = fn(epi, bn, splits, ptr(a_d), ptr(w_d), ptr(got), ptr(got) if epi & jc.EPI_RES else None,
                ptr(st_d), ptr(cs_d), ptr(got_st), None, 0, m, n, k, 1e-5, ptr(rope_d), None,
                stream)
        assert rc == 0, lib.jc_last_error()
        torch.cuda.synchronize()
        assert jc.device_error() == 0
        got_h = host_u16(got)
        e, el = rel_err(O.f32(got_h), O.f32(want)), elem_err(O.f32(got_h), O.f32(want))
        assert e < 1e-3 and el < 1e-2, f"call {call}: rel err {e:.2e}, worst element {el:.2e}"
        # Same configuration as jc_gemm, same arithmetic order: the same bits.
        assert np.array_equal(got_h, ref_h), f"call {call}: differs from jc_gemm"
        if epi & jc.EPI_STATS:
            x = O.f32(got_h).astype(np.float64)
            st = got_st.cpu().numpy().reshape(-1, 2).astype(np.float64)
            q = np.maximum((x * x).sum(1), 1e-30)
            se = np.max(np.maximum(np.abs(st[:, 0] - x.sum(1)) / np.sqrt(q), np.abs(st[:, 1] - q) / q))
            assert se < 1e-4, f"call {call}: stats err {se:.2e}"


def test_noalloc_rejects_scratch_overflow(noalloc):
    jc, O, lib, fn = noalloc
    m, n, k = 1024, 2304, 2048
    a = torch.zeros(m, k, device="cuda").half()
    w = torch.zeros(n, k, device="cuda").half()
    c = torch.zeros(m, n, device="cuda").half()
    rc = fn(0, 64, 8, ptr(a), ptr(w), ptr(c), None, None, None, None, None, 0, m, n, k, 1e-5, None,
            None, torch.cuda.current_stream().cuda_stream)
    assert rc == -1 and b"scratch" in lib.jc_last_error()
