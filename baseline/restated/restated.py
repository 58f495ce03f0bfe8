"""ctypes binding of librestated.so: the reference's per-step GPU forward restated in CUDA C++
(restated.cu), the latency baseline the package is compared with on the same GPU."""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librestated.so")
SYMBOLS = ("jc_restated_load", "jc_restated_run", "jc_restated_free")
_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is not built (make -C {HERE})")
        L = ctypes.CDLL(LIB_PATH)
        L.jc_restated_load.restype = ctypes.c_void_p
        L.jc_restated_load.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                       ctypes.c_size_t, ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t]
        L.jc_restated_run.restype = ctypes.c_int
        L.jc_restated_run.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                      ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint32,
                                      ctypes.c_void_p, ctypes.c_void_p, ctypes.c_char_p,
                                      ctypes.c_size_t]
        L.jc_restated_free.restype = None
        L.jc_restated_free.argtypes = [ctypes.c_void_p]
        u32, P = ctypes.c_uint32, ctypes.c_void_p
        for f in ("jc_restated_gemm_ws_floats", "jc_restated_gemm_counters"):
            getattr(L, f).restype = ctypes.c_size_t
            getattr(L, f).argtypes = [u32, u32, u32, ctypes.c_int]
        L.jc_restated_gemm.restype = ctypes.c_int
        L.jc_restated_gemm.argtypes = [u32, P, P, P, P, P, P, P, P, P, P, u32, u32, u32, u32,
                                       ctypes.c_float, P, P, ctypes.c_int, P]
        L.jc_restated_attention.restype = ctypes.c_int
        L.jc_restated_attention.argtypes = [P, P, u32, u32, u32, P]
        _lib = L
    return _lib


class Restated:
    """The restated reference forward on GPU `device` from raw weights (cfg: the package's
    jc_model_config ctypes structure; raw: float32 array of julia_cuda_raw_size values)."""

    def __init__(self, cfg, raw, max_length=0, device=0):
        raw = np.ascontiguousarray(raw, dtype=np.float32)
        err = ctypes.create_string_buffer(512)
        self._cfg = cfg
        self.h = lib().jc_restated_load(ctypes.byref(cfg), raw.ctypes.data, raw.size, max_length,
                                        device, err, 512)
        if not self.h:
            raise RuntimeError(err.value.decode())

    def run(self, ids, markers, qtype=0):
        """(logits float32 [len(markers)], GPU ms embed -> logits)."""
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        markers = np.ascontiguousarray(markers, dtype=np.uint32)
        out = np.zeros(markers.size, np.float32)
        ms = ctypes.c_float()
        err = ctypes.create_string_buffer(512)
        rc = lib().jc_restated_run(self.h, ids.ctypes.data, ids.size, markers.ctypes.data,
                                   markers.size, qtype, out.ctypes.data, ctypes.byref(ms), err, 512)
        if rc != 0:
            raise RuntimeError(err.value.decode())
        return out, ms.value

    def close(self):
        if self.h:
            lib().jc_restated_free(self.h)
            self.h = None


def _p(t):
    return None if t is None else t.data_ptr()


def gemm_scratch(torch, m, n, k, sms):
    """Split-K workspace and zeroed counters for one restated GEMM shape (None when unsplit)."""
    wf = lib().jc_restated_gemm_ws_floats(m, n, k, sms)
    if not wf:
        return None, None
    cnt = lib().jc_restated_gemm_counters(m, n, k, sms)
    return (torch.empty(wf, dtype=torch.float32, device="cuda"),
            torch.zeros(cnt, dtype=torch.int32, device="cuda"))


def gemm(torch, epi, a, w, c, sms, res=None, ws=None, counters=None, stats_in=None, colsum=None,
         stats_out=None, zero=None, eps=1e-5, rope=None, bias=None):
    """One restated GEMM on torch tensors, queued on torch's current stream. rope: the natural
    [rows][32][2] f32 table."""
    m, k = a.shape
    n = w.shape[0]
    rc = lib().jc_restated_gemm(epi, _p(a), _p(w), _p(c), _p(res), _p(ws), _p(counters),
                                _p(stats_in), _p(colsum), _p(stats_out), _p(zero),
                                0 if zero is None else zero.numel(), m, n, k, eps, _p(rope),
                                _p(bias), sms, torch.cuda.current_stream().cuda_stream)
    if rc != 0:
        raise RuntimeError("restated gemm: bad arguments or launch failure")


def attention(torch, qkv, o, window):
    """The restated attention (one key range, as the reference's per-step launch)."""
    n, d = o.shape
    rc = lib().jc_restated_attention(_p(qkv), _p(o), n, window, d,
                                     torch.cuda.current_stream().cuda_stream)
    if rc != 0:
        raise RuntimeError("restated attention: bad arguments or launch failure")
