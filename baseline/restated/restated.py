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
