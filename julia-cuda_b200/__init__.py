"""julia-cuda-b200: the julia-cuda encoder hot path on B200, from Python.

A thin ctypes layer over libjulia_cuda.so (include/julia_cuda.h), mirroring the reference's own
FFI surface: the engine calls of src/capi.rs (julia_cuda_load / run / free / device / tier) and the
kernel-level launches of src/gemm.rs, src/attn.rs and src/lib.rs. torch tensors are used only for
device memory and streams. There is no CPU fallback: importing this package on a machine without
the built library raises, and every kernel call fails loudly if its launch fails.

The directory name is not an identifier; import it with importlib.import_module("julia-cuda_b200").
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libjulia_cuda.so")

EPI_RES, EPI_GEGLU, EPI_LN, EPI_STATS = 1, 2, 4, 8
EPI_ROPE, EPI_BIAS, EPI_RELU, EPI_GELU = 16, 32, 64, 128

# The reference's eight GEMM variants (src/gemm.rs:57-87) as epilogue flags.
EPILOGUES = {
    "rope": EPI_ROPE,
    "lnrope": EPI_LN | EPI_ROPE,
    "lngeglu": EPI_LN | EPI_GEGLU,
    "resstats": EPI_RES | EPI_STATS,
    "lnbias": EPI_LN | EPI_BIAS,
    "lnbiasrelu": EPI_LN | EPI_BIAS | EPI_RELU,
    "lnbiasgelu": EPI_LN | EPI_BIAS | EPI_GELU,
    "biasresstats": EPI_BIAS | EPI_RES | EPI_STATS,
}


class JuliaCudaError(RuntimeError):
    pass


class LaunchInfo(ctypes.Structure):
    """jc_launch_info: one launch of a profiled forward."""

    _fields_ = [("kind", ctypes.c_uint32), ("epi", ctypes.c_uint32), ("m", ctypes.c_uint32),
                ("n", ctypes.c_uint32), ("k", ctypes.c_uint32), ("layer", ctypes.c_int32),
                ("ctas", ctypes.c_uint32), ("tile", ctypes.c_uint32), ("record", ctypes.c_uint32),
                ("launch", ctypes.c_uint32), ("records", ctypes.c_uint32), ("items", ctypes.c_uint32)]


LAUNCH_KINDS = {0: "gemm", 1: "attention", 2: "embed", 3: "head input", 4: "gather", 5: "score",
                6: "copy"}


class Config(ctypes.Structure):
    """jc_model_config."""

    _fields_ = [
        ("d_model", ctypes.c_int32), ("n_heads", ctypes.c_int32), ("inter", ctypes.c_int32),
        ("n_layers", ctypes.c_int32), ("vocab", ctypes.c_int32), ("head_ff", ctypes.c_int32),
        ("scorer_hidden", ctypes.c_int32), ("n_head_layers", ctypes.c_int32),
        ("global_every", ctypes.c_int32), ("window", ctypes.c_int32),
        ("max_positions", ctypes.c_int32), ("n_qtypes", ctypes.c_int32),
        ("norm_eps", ctypes.c_float), ("head_eps", ctypes.c_float),
        ("theta_global", ctypes.c_float), ("theta_local", ctypes.c_float),
    ]

    def replace(self, **kw) -> "Config":
        c = Config()
        ctypes.memmove(ctypes.byref(c), ctypes.byref(self), ctypes.sizeof(Config))
        for k, v in kw.items():
            setattr(c, k, v)
        if "d_model" in kw and "n_heads" not in kw:
            c.n_heads = c.d_model // 64
        return c


def build() -> None:
    """Compiles libjulia_cuda.so in place (nvcc -gencode arch=compute_100a,code=sm_100a)."""
    subprocess.run(["make", "-s", "-j8", "-C", HERE], check=True)


_lib = None


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise JuliaCudaError(f"{LIB_PATH} is not built (run build() / make -C julia-cuda_b200)")
    L = ctypes.CDLL(LIB_PATH)
    P, u32, i32, f32, sz, u64 = (ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int, ctypes.c_float,
                                 ctypes.c_size_t, ctypes.c_uint64)
    cfgp = ctypes.POINTER(Config)
    ch = ctypes.c_char_p
    sig = {
        "julia_cuda_tier": ([], ch),
        "julia_cuda_load": ([ch, sz, P, sz], P),
        "julia_cuda_free": ([P], None),
        "julia_cuda_device": ([P, P, sz], None),
        "julia_cuda_run": ([P, sz, P, P, P, P, P, i32, P, P, P, sz], i32),
        "julia_cuda_default_config": ([cfgp], None),
        "julia_cuda_raw_size": ([cfgp], sz),
        "julia_cuda_raw_offsets": ([cfgp, P, sz], i32),
        "julia_cuda_init_random": ([cfgp, u64, P], None),
        "julia_cuda_save_raw": ([ch, cfgp, P, P, sz], i32),
        "julia_cuda_load_raw": ([cfgp, P, sz, sz, i32, P, sz], P),
        "julia_cuda_load_random": ([cfgp, u64, sz, i32, P, sz], P),
        "julia_cuda_forward_device": ([P, P, u32, P, u32, u32, i32, P, P, P, P, sz], i32),
        "julia_cuda_forward_trace": ([P, P, u32, P, u32, u32, i32, P, P, P, P, P, P, sz], i32),
        "julia_cuda_forward_profile": ([P, P, u32, P, u32, u32, P, P, u32, P, sz, P, P, P, sz], i32),
        "julia_cuda_forward_profile_mode": ([P, P, u32, P, u32, u32, i32, P, P, u32, P, sz, P, P, P, sz],
                                            i32),
        "julia_cuda_launches_per_forward": ([P, u32, u32, i32], i32),
        "julia_cuda_set_head_length": ([P, sz], i32),
        "julia_cuda_set_packing": ([P, sz], i32),
        "julia_cuda_barrier_timeout_probe": ([P, u64, P, P, sz], i32),
        "julia_cuda_device_error": ([P, P, P, sz], i32),
        "julia_cuda_engine_config": ([P, cfgp, P, P, P], i32),
        "julia_cuda_read_checkpoint": ([ch, cfgp, P, sz, P, P, sz], i32),
        "julia_cuda_save_checkpoint": ([ch, cfgp, P, i32, P, sz], i32),
        "julia_cuda_prepare_host": ([cfgp, P, sz, sz, P, sz, P, sz, P, P, P, sz], i32),
        "jc_gemm": ([u32, i32, i32, P, P, P, P, P, P, P, P, P, P, u32, u32, u32, u32, f32, P, P, P],
                    i32),
        "jc_layer": ([P, P, P, P, P, P, P, P, P, u32, P, P, P, P, u32, u32, u32, u32, f32, u32, P],
                     i32),
        "jc_gemm_ws_floats": ([u32, u32, u32, i32, i32], sz),
        "jc_gemm_counters": ([u32, u32, u32, i32, i32], sz),
        "jc_choose_gemm": ([u32, u32, u32, i32, P, P], i32),
        "jc_attention": ([P, P, u32, u32, u32, u32, P, P, P], i32),
        "jc_attention_ws_floats": ([u32, u32, u32], sz),
        "jc_attention_counters": ([u32, u32], sz),
        "jc_attention_tc_min": ([P, P], None),
        "jc_gemm_tile_rows": ([P], None),
        "jc_gemm_pair_policy": ([P], None),
        "jc_persist_tile": ([u32, u32, u32, u32, u32], i32),
        "jc_gemm_phase_us": ([u32, u32, u32, i32, u32], ctypes.c_double),
        "jc_persist_phase_us": ([u32, u32, u32, i32, u32], ctypes.c_double),
        "jc_persist_tile_policy": ([P], None),
        "jc_embed": ([P, u32, P, P, u32, f32, P, P, P], i32),
        "jc_norm_add": ([P, u32, u32, P, P, f32, P, P, P], i32),
        "jc_score": ([P, u32, P, f32, P, u32, P, P], i32),
        "jc_last_error": ([], ch),
        "jc_device_error": ([P], i32),
        "jc_prep_fold_layernorm": ([P, P, u32, u32, P, P], None),
        "jc_prep_fold_layernorm_bias": ([P, P, P, P, u32, u32, P, P, P], None),
        "jc_prep_interleave_geglu_f16": ([P, u32, u32, P], None),
        "jc_prep_interleave_geglu_f32": ([P, u32, u32, P], None),
        "jc_prep_rope_table": ([f32, u32, P], None),
        "jc_prep_rope_gemm": ([P, u32, P], None),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


def last_error() -> str:
    return lib().jc_last_error().decode(errors="replace")


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise JuliaCudaError(f"{what}: {last_error()}")


def default_config(**kw) -> Config:
    c = Config()
    lib().julia_cuda_default_config(ctypes.byref(c))
    return c.replace(**kw) if kw else c


def _np_ptr(a):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def _t_ptr(t):
    """Device pointer of a contiguous torch tensor (or None)."""
    if t is None:
        return None
    if not t.is_contiguous():
        raise JuliaCudaError("tensors passed to the kernels must be contiguous")
    return t.data_ptr()


def _stream(stream):
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return getattr(stream, "cuda_stream", stream)


# ------------------------------------------------------------------------------------------------
# raw model format and host preparation

def raw_size(cfg: Config) -> int:
    return lib().julia_cuda_raw_size(ctypes.byref(cfg))


def raw_offsets(cfg: Config) -> np.ndarray:
    cap = 16 * (cfg.n_layers + cfg.n_head_layers) + 64
    out = np.zeros(cap, np.uint64)
    n = lib().julia_cuda_raw_offsets(ctypes.byref(cfg), _np_ptr(out), cap)
    if n < 0:
        raise JuliaCudaError(last_error())
    return out[:n]


def read_checkpoint(directory: str):
    """(Config, raw f32 weights) of a checkpoint directory (julia_cuda_read_checkpoint)."""
    cfg = Config()
    n = ctypes.c_size_t(0)
    err = ctypes.create_string_buffer(1024)
    if lib().julia_cuda_read_checkpoint(directory.encode(), ctypes.byref(cfg), None, 0,
                                        ctypes.byref(n), err, 1024) != 0:
        raise JuliaCudaError(err.value.decode(errors="replace"))
    raw = np.empty(n.value, np.float32)
    if lib().julia_cuda_read_checkpoint(directory.encode(), ctypes.byref(cfg), _np_ptr(raw),
                                        raw.size, None, err, 1024) != 0:
        raise JuliaCudaError(err.value.decode(errors="replace"))
    return cfg, raw


def save_checkpoint(directory: str, cfg: Config, raw: np.ndarray, dtype: int = 0) -> None:
    """Writes a checkpoint directory (julia_cuda_save_checkpoint; dtype 0 F32, 1 F16, 2 BF16)."""
    raw = np.ascontiguousarray(raw, np.float32)
    err = ctypes.create_string_buffer(1024)
    if lib().julia_cuda_save_checkpoint(directory.encode(), ctypes.byref(cfg), _np_ptr(raw), dtype,
                                        err, 1024) != 0:
        raise JuliaCudaError(err.value.decode(errors="replace"))


def prepare_host(cfg: Config, raw: np.ndarray, max_length: int = 0):
    """The prepared f16 (bit patterns) and f32 arenas an engine uploads (julia_cuda_prepare_host)."""
    raw = np.ascontiguousarray(raw, np.float32)
    n16, n32 = ctypes.c_size_t(0), ctypes.c_size_t(0)
    err = ctypes.create_string_buffer(1024)
    args = (ctypes.byref(cfg), _np_ptr(raw), raw.size, max_length)
    if lib().julia_cuda_prepare_host(*args, None, 0, None, 0, ctypes.byref(n16), ctypes.byref(n32),
                                     err, 1024) != 0:
        raise JuliaCudaError(err.value.decode(errors="replace"))
    a16, a32 = np.empty(n16.value, np.uint16), np.empty(n32.value, np.float32)
    if lib().julia_cuda_prepare_host(*args, _np_ptr(a16), a16.size, _np_ptr(a32), a32.size, None,
                                     None, err, 1024) != 0:
        raise JuliaCudaError(err.value.decode(errors="replace"))
    return a16, a32


def init_random(cfg: Config, seed: int) -> np.ndarray:
    raw = np.empty(raw_size(cfg), np.float32)
    lib().julia_cuda_init_random(ctypes.byref(cfg), seed, _np_ptr(raw))
    return raw


def prep_fold_layernorm(w: np.ndarray, gamma: np.ndarray):
    out, k = w.shape
    w16 = np.zeros((out, k), np.uint16)
    cs = np.zeros(out, np.float32)
    lib().jc_prep_fold_layernorm(_np_ptr(np.ascontiguousarray(w, np.float32)),
                                 _np_ptr(np.ascontiguousarray(gamma, np.float32)), out, k,
                                 _np_ptr(w16), _np_ptr(cs))
    return w16, cs


def prep_fold_layernorm_bias(w, gamma, beta, b):
    out, k = w.shape
    w16 = np.zeros((out, k), np.uint16)
    cs = np.zeros(out, np.float32)
    bias = np.zeros(out, np.float32)
    f = lambda a: _np_ptr(np.ascontiguousarray(a, np.float32))
    lib().jc_prep_fold_layernorm_bias(f(w), f(gamma), f(beta), f(b), out, k, _np_ptr(w16),
                                      _np_ptr(cs), _np_ptr(bias))
    return w16, cs, bias


def prep_interleave_geglu(w: np.ndarray) -> np.ndarray:
    """Wi rows (GELU inputs, then gates) in the GeGLU epilogue's order; 1-D: a vector."""
    a = np.ascontiguousarray(w)
    n = a.shape[0]
    k = a.shape[1] if a.ndim == 2 else 1
    out = np.empty_like(a)
    if a.dtype == np.uint16:
        lib().jc_prep_interleave_geglu_f16(_np_ptr(a), n, k, _np_ptr(out))
    elif a.dtype == np.float32:
        lib().jc_prep_interleave_geglu_f32(_np_ptr(a), n, k, _np_ptr(out))
    else:
        raise JuliaCudaError("interleave: uint16 (f16 bits) or float32 only")
    return out


def prep_rope_table(theta: float, n: int) -> np.ndarray:
    t = np.zeros((n, 32, 2), np.float32)
    lib().jc_prep_rope_table(theta, n, _np_ptr(t))
    return t


def prep_rope_gemm(table: np.ndarray, m: int) -> np.ndarray:
    """jc_gemm's RoPE argument (float4 [16][m]) from a [>= m][32][2] (cos, sin) table."""
    t = np.ascontiguousarray(table, np.float32)
    assert t.shape[0] >= m and t.shape[1:] == (32, 2)
    out = np.zeros((16, m, 4), np.float32)
    lib().jc_prep_rope_gemm(_np_ptr(t), m, _np_ptr(out))
    return out


# ------------------------------------------------------------------------------------------------
# kernels on torch device tensors (f16 tensors are torch.float16)

def gemm_scratch(m: int, n: int, k: int, bn: int = 0, splits: int = 0, device="cuda"):
    """Split-K workspace and zeroed counters for jc_gemm with this shape / configuration."""
    import torch
    ws = lib().jc_gemm_ws_floats(m, n, k, bn, splits)
    cnt = lib().jc_gemm_counters(m, n, k, bn, splits)
    return (torch.empty(max(ws, 1), dtype=torch.float32, device=device),
            torch.zeros(max(cnt, 1), dtype=torch.int32, device=device))


def gemm(epi: int, a, w, c, *, res=None, stats_in=None, colsum=None, stats_out=None, zero=None,
         eps: float = 1e-5, rope=None, bias=None, bn: int = 0, splits: int = 0, ws=None,
         counters=None, stream=None) -> None:
    """c = epilogue(a . w^T) (jc_gemm); a [m, k], w [n, k] f16."""
    m, k = a.shape
    n = w.shape[0]
    if ws is None or counters is None:
        ws, counters = gemm_scratch(m, n, k, bn, splits, a.device)
    rc = lib().jc_gemm(epi, bn, splits, _t_ptr(a), _t_ptr(w), _t_ptr(c), _t_ptr(res), _t_ptr(ws),
                       _t_ptr(counters), _t_ptr(stats_in), _t_ptr(colsum), _t_ptr(stats_out),
                       _t_ptr(zero), 0 if zero is None else zero.numel(), m, n, k, eps,
                       _t_ptr(rope), _t_ptr(bias), _stream(stream))
    _check(rc, "jc_gemm")


def layer(x, qkv, o, mbuf, stats_attn, stats_mlp, wqkv, qkv_colsum, rope, wo, wi, wi_colsum,
          wo_mlp, heads: int, eps: float = 1e-5, window: int = 0, rope_stride: int = 0,
          stream=None) -> None:
    """One encoder layer on the persistent kernel (jc_layer): x [m, d] f16 updated in place;
    qkv, o, mbuf scratch; stats_mlp x's row statistics in and out, stats_attn scratch;
    qkv_colsum None for a layer without LayerNorm before qkv. rope in jc_gemm's layout."""
    m, d = x.shape
    inter = mbuf.shape[1]
    rc = lib().jc_layer(_t_ptr(x), _t_ptr(qkv), _t_ptr(o), _t_ptr(mbuf), _t_ptr(stats_attn),
                        _t_ptr(stats_mlp), _t_ptr(wqkv), _t_ptr(qkv_colsum), _t_ptr(rope),
                        rope_stride, _t_ptr(wo), _t_ptr(wi), _t_ptr(wi_colsum), _t_ptr(wo_mlp),
                        m, d, heads, inter, eps, window, _stream(stream))
    _check(rc, "jc_layer")


def attention(qkv, o, heads: int, window: int = 0, kv_chunks: int = 0, stream=None, ws=None,
              counters=None) -> None:
    """o = softmax(q k^T / 8) v per head (jc_attention). ws / counters: split-KV scratch sized for
    16 key ranges (allocated here when not given)."""
    import torch
    n = qkv.shape[0]
    chunks = kv_chunks
    cnt = counters
    if kv_chunks != 1 and (ws is None or cnt is None):
        probe = 16 if kv_chunks == 0 else kv_chunks
        ws = torch.empty(max(lib().jc_attention_ws_floats(n, heads, probe), 1), dtype=torch.float32,
                         device=qkv.device)
        cnt = torch.zeros(max(lib().jc_attention_counters(n, heads), 1), dtype=torch.int32,
                          device=qkv.device)
    rc = lib().jc_attention(_t_ptr(qkv), _t_ptr(o), n, heads, window, chunks, _t_ptr(ws),
                            _t_ptr(cnt), _stream(stream))
    _check(rc, "jc_attention")


def gemm_tile_rows(rows: int) -> int:
    """Sets the GEMM tile height policy (0 automatic, 128, or 64 wherever legal;
    jc_gemm_tile_rows); returns the previous one."""
    r = ctypes.c_int(rows)
    lib().jc_gemm_tile_rows(ctypes.byref(r))
    return r.value


def gemm_pair_policy(policy: int) -> int:
    """Sets the CTA-pair GEMM policy (1 every unsplit 128/256-column launch, 0 automatic: the
    persistent 256-column launches, -1 never; jc_gemm_pair_policy); returns the previous one (-2:
    not a policy, nothing changed)."""
    r = ctypes.c_int(policy)
    lib().jc_gemm_pair_policy(ctypes.byref(r))
    return r.value


def persist_tile_policy(bn: int) -> int:
    """Sets the persistent kernel's tile width policy (0 the plan, 32 or 64;
    jc_persist_tile_policy) for later-planned launches; returns the previous one (-1: not a
    policy, nothing changed)."""
    r = ctypes.c_int(bn)
    lib().jc_persist_tile_policy(ctypes.byref(r))
    return r.value


def attention_tc_min(global_min: int, window_min: int) -> tuple:
    """Sets the shortest global / sliding-window sequence for the tcgen05 attention kernel
    (jc_attention_tc_min); returns the previous pair."""
    g, w = ctypes.c_uint32(global_min), ctypes.c_uint32(window_min)
    lib().jc_attention_tc_min(ctypes.byref(g), ctypes.byref(w))
    return g.value, w.value


def embed(ids, table, gamma, x, eps=1e-5, stats=None, stream=None) -> None:
    rc = lib().jc_embed(_t_ptr(ids), ids.numel(), _t_ptr(table), _t_ptr(gamma), table.shape[1],
                        eps, _t_ptr(x), _t_ptr(stats), _stream(stream))
    _check(rc, "jc_embed")


def norm_add(x, gamma, add, out, stats, eps=1e-5, stream=None) -> None:
    n, d = x.shape
    rc = lib().jc_norm_add(_t_ptr(x), n, d, _t_ptr(gamma), _t_ptr(add), eps, _t_ptr(out),
                           _t_ptr(stats), _stream(stream))
    _check(rc, "jc_norm_add")


def score(y, w, b: float, markers, logits, stream=None) -> None:
    rc = lib().jc_score(_t_ptr(y), y.shape[1], _t_ptr(w), b, _t_ptr(markers), markers.numel(),
                        _t_ptr(logits), _stream(stream))
    _check(rc, "jc_score")


def device_error() -> int:
    code = ctypes.c_uint32(0)
    _check(lib().jc_device_error(ctypes.byref(code)), "jc_device_error")
    return code.value


# ------------------------------------------------------------------------------------------------
# engine (the reference's Engine / C ABI)

class Engine:
    """One model on one GPU: julia_cuda_load_raw / julia_cuda_load_random + julia_cuda_run."""

    def __init__(self, handle, cfg: Config):
        self._h = handle
        self.cfg = cfg

    @classmethod
    def load_raw(cls, cfg: Config, raw: np.ndarray, max_length: int = 1024, device: int = 0):
        raw = np.ascontiguousarray(raw, np.float32)
        err = ctypes.create_string_buffer(1024)
        h = lib().julia_cuda_load_raw(ctypes.byref(cfg), _np_ptr(raw), raw.size, max_length,
                                      device, err, 1024)
        if not h:
            raise JuliaCudaError(err.value.decode(errors="replace"))
        return cls(h, cfg)

    @classmethod
    def load_random(cls, cfg: Config, seed: int, max_length: int = 1024, device: int = 0):
        err = ctypes.create_string_buffer(1024)
        h = lib().julia_cuda_load_random(ctypes.byref(cfg), seed, max_length, device, err, 1024)
        if not h:
            raise JuliaCudaError(err.value.decode(errors="replace"))
        return cls(h, cfg)

    @classmethod
    def load(cls, directory: str, max_length: int = 0):
        err = ctypes.create_string_buffer(1024)
        h = lib().julia_cuda_load(directory.encode(), max_length, err, 1024)
        if not h:
            raise JuliaCudaError(err.value.decode(errors="replace"))
        cfg = Config()
        lib().julia_cuda_engine_config(h, ctypes.byref(cfg), None, None, None)
        return cls(h, cfg)

    def close(self) -> None:
        if self._h:
            lib().julia_cuda_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def device_name(self) -> str:
        buf = ctypes.create_string_buffer(256)
        lib().julia_cuda_device(self._h, buf, 256)
        return buf.value.decode()

    def _staging(self, n_ids: int, n_mk: int, b: int):
        """Per-engine argument arrays for julia_cuda_run, grown on demand; their addresses are
        taken once (numpy's .ctypes costs microseconds a call, a sizeable share of a request)."""
        st = getattr(self, "_st", None)
        if st is None or st["ids"].size < n_ids or st["mk"].size < max(n_mk, 1) or st["lens"].size < b:
            cap = lambda x, old: max(x, 2 * old)  # noqa: E731
            old = st or {"ids": np.zeros(0), "mk": np.zeros(0), "lens": np.zeros(0)}
            st = {"ids": np.zeros(cap(n_ids, old["ids"].size), np.uint32),
                  "mk": np.zeros(cap(max(n_mk, 1), old["mk"].size), np.uint32),
                  "logits": np.zeros(cap(max(n_mk, 1), old["mk"].size), np.float32)}
            nb = cap(b, old["lens"].size)
            st.update(lens=np.zeros(nb, np.uint64), nmk=np.zeros(nb, np.uint64),
                      qt=np.zeros(nb, np.uint32), gpu_ms=np.zeros(nb, np.float32),
                      err=ctypes.create_string_buffer(1024))
            st["ptr"] = {k: v.ctypes.data for k, v in st.items() if isinstance(v, np.ndarray)}
            self._st = st
        return st

    def run(self, seqs, layer_fused: int = 0):
        """seqs: list of (ids, markers, qtype). Returns (list of logits arrays, gpu_ms array).
        layer_fused: 0 per-step kernels, 1 one persistent launch per layer, 2 whole model."""
        b = len(seqs)
        n_ids = sum(len(s[0]) for s in seqs)
        n_mk = sum(len(s[1]) for s in seqs)
        st = self._staging(n_ids, n_mk, b)
        at_i = at_m = 0
        for i, (ids, mk, qt) in enumerate(seqs):
            n, k = len(ids), len(mk)
            st["ids"][at_i:at_i + n] = ids
            st["mk"][at_m:at_m + k] = mk
            st["lens"][i], st["nmk"][i], st["qt"][i] = n, k, qt
            at_i += n
            at_m += k
        ptr = st["ptr"]
        rc = lib().julia_cuda_run(self._h, b, ptr["ids"], ptr["lens"], ptr["mk"], ptr["nmk"],
                                  ptr["qt"], int(layer_fused), ptr["logits"], ptr["gpu_ms"],
                                  st["err"], 1024)
        if rc != 0:
            raise JuliaCudaError(st["err"].value.decode(errors="replace"))
        out, at = [], 0
        logits = st["logits"]
        for s in seqs:
            k = len(s[1])
            out.append(logits[at:at + k].copy())
            at += k
        return out, st["gpu_ms"][:b].copy()

    def forward_device(self, ids, markers, qtype: int, logits, trace=None, layer_fused=False,
                       stream=None) -> None:
        err = ctypes.create_string_buffer(1024)
        rc = lib().julia_cuda_forward_device(self._h, _t_ptr(ids), ids.numel(), _t_ptr(markers),
                                             markers.numel(), qtype, int(layer_fused),
                                             _t_ptr(logits), _t_ptr(trace), _stream(stream), err,
                                             1024)
        if rc != 0:
            raise JuliaCudaError(err.value.decode(errors="replace"))

    def forward_trace(self, ids, markers, qtype: int, logits, trace=None, head_trace=None,
                      scorer_trace=None, layer_fused=False, stream=None) -> None:
        """forward_device with the head and the scorer traced too (julia_cuda_forward_trace):
        trace [n_layers][n][D], head_trace [n_head_layers + 1][nh][D], scorer_trace
        [n_markers][scorer_hidden], f16 device tensors, each optional."""
        err = ctypes.create_string_buffer(1024)
        rc = lib().julia_cuda_forward_trace(self._h, _t_ptr(ids), ids.numel(), _t_ptr(markers),
                                            markers.numel(), qtype, int(layer_fused),
                                            _t_ptr(logits), _t_ptr(trace), _t_ptr(head_trace),
                                            _t_ptr(scorer_trace), _stream(stream), err, 1024)
        if rc != 0:
            raise JuliaCudaError(err.value.decode(errors="replace"))

    def forward_profile(self, ids, markers, qtype: int, logits, records_per_launch: int = 1024,
                        stream=None, layer_fused: int = 0):
        """A forward with phase stamps (julia_cuda_forward_profile_mode): per CTA for the
        per-step kernels, per work item for the persistent kernel (layer_fused 1 or 2). Returns
        (records uint64 [n, 8], list of launch dicts; entry e owns records[e["record"]:
        e["record"] + e["records"]]). A per-step record holds %globaltimer ns at entry, inputs
        ready, first stage, results complete, outputs written, exit; an item's at item taken,
        inputs ready, first stage, results complete, outputs written, reported (0 where a stage
        does not apply); then the SM and the CTA index."""
        import torch
        cap = 4 * (self.cfg.n_layers + self.cfg.n_head_layers) * 6 + 64
        prof = torch.zeros(cap * records_per_launch * 8, dtype=torch.int64, device=ids.device)
        info = (LaunchInfo * cap)()
        n = ctypes.c_size_t(0)
        err = ctypes.create_string_buffer(1024)
        rc = lib().julia_cuda_forward_profile_mode(self._h, _t_ptr(ids), ids.numel(),
                                                   _t_ptr(markers), markers.numel(), qtype,
                                                   int(layer_fused), _t_ptr(logits), _t_ptr(prof),
                                                   records_per_launch, info, cap, ctypes.byref(n),
                                                   _stream(stream), err, 1024)
        if rc != 0:
            raise JuliaCudaError(err.value.decode(errors="replace"))
        launches = [{f: getattr(info[i], f) for f, _ in LaunchInfo._fields_} for i in range(n.value)]
        recs = prof.view(-1, 8).cpu().numpy().view(np.uint64)
        return recs, launches

    def set_packing(self, rows: int) -> None:
        """run() packs consecutive requests into forwards of up to `rows` tokens (0: off)."""
        if lib().julia_cuda_set_packing(self._h, rows) != 0:
            raise JuliaCudaError("set_packing: no engine, or rows above max_length")

    def set_head_length(self, rows: int) -> None:
        """The head runs on the first `rows` rows of later requests (0: all rows)."""
        if lib().julia_cuda_set_head_length(self._h, rows) != 0:
            raise JuliaCudaError("set_head_length: no engine")

    def launches_per_forward(self, n: int, n_markers: int, layer_fused=False) -> int:
        return lib().julia_cuda_launches_per_forward(self._h, n, n_markers, int(layer_fused))

    def barrier_timeout_probe(self, timeout_ns: int) -> int:
        """Makes a persistent-kernel grid barrier time out on purpose; returns the device error
        code the kernel recorded (4: a grid barrier timed out)."""
        code = ctypes.c_uint32(0)
        err = ctypes.create_string_buffer(1024)
        rc = lib().julia_cuda_barrier_timeout_probe(self._h, timeout_ns, ctypes.byref(code), err,
                                                   1024)
        if rc != 0:
            raise JuliaCudaError(err.value.decode(errors="replace"))
        return code.value

    def device_error(self) -> int:
        """Waits for the engine's stream and reads (and clears) the engine's own device error
        word (julia_cuda_device_error; 0: none)."""
        code = ctypes.c_uint32(0)
        err = ctypes.create_string_buffer(1024)
        rc = lib().julia_cuda_device_error(self._h, ctypes.byref(code), err, 1024)
        if rc != 0:
            raise JuliaCudaError(err.value.decode(errors="replace"))
        return code.value
