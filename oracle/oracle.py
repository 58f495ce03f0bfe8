"""ctypes wrapper of the CPU oracle (liboracle.so). TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import this module, as the
checker or the timed CPU baseline. The product (julia-cuda_b200/) never does. The C sources
(oracle.c / oracle.h) say which reference function each piece restates.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

OR_RES, OR_GEGLU, OR_LN, OR_STATS, OR_ROPE, OR_BIAS, OR_RELU, OR_GELU = 1, 2, 4, 8, 16, 32, 64, 128


class Config(ctypes.Structure):
    _fields_ = [
        ("d_model", ctypes.c_int32), ("n_heads", ctypes.c_int32), ("inter", ctypes.c_int32),
        ("n_layers", ctypes.c_int32), ("vocab", ctypes.c_int32), ("head_ff", ctypes.c_int32),
        ("scorer_hidden", ctypes.c_int32), ("n_head_layers", ctypes.c_int32),
        ("global_every", ctypes.c_int32), ("window", ctypes.c_int32),
        ("max_positions", ctypes.c_int32), ("n_qtypes", ctypes.c_int32),
        ("norm_eps", ctypes.c_float), ("head_eps", ctypes.c_float),
        ("theta_global", ctypes.c_float), ("theta_local", ctypes.c_float),
    ]


def config(d_model=768, inter=1152, n_layers=22, vocab=50368, head_ff=2048, scorer_hidden=384,
           n_head_layers=2, global_every=3, window=64, max_positions=8192, n_qtypes=3,
           norm_eps=1e-5, head_eps=1e-5, theta_global=160000.0, theta_local=10000.0) -> Config:
    """The benchmark's model (hidden 768, 12 heads, 22 layers); keyword overrides for tests."""
    return Config(d_model, d_model // 64, inter, n_layers, vocab, head_ff, scorer_hidden,
                  n_head_layers, global_every, window, max_positions, n_qtypes, norm_eps,
                  head_eps, theta_global, theta_local)


def reference_width_config(**kw) -> Config:
    """The reference's own Julia-1 width: hidden 384, 6 heads, scorer D -> D -> 1."""
    base = dict(d_model=384, inter=1152, scorer_hidden=384)
    base.update(kw)
    return config(**base)


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.c_void_p
        i32, u64, f32, sz = ctypes.c_int, ctypes.c_uint64, ctypes.c_float, ctypes.c_size_t
        cfgp = ctypes.POINTER(Config)
        L.or_raw_size.argtypes = [cfgp]
        L.or_raw_size.restype = sz
        L.or_init_random.argtypes = [cfgp, u64, P]
        L.or_fill_normal.argtypes = [P, sz, u64, f32, f32]
        L.or_forward_f32_head.argtypes = [cfgp, P, P, i32, P, i32, i32, i32, P, P]
        L.or_forward_f32_head.restype = i32
        L.or_forward_emu_head.argtypes = [cfgp, P, P, i32, P, i32, i32, i32, P, P, i32]
        L.or_forward_emu_head.restype = i32
        L.or_forward_f32_full.argtypes = [cfgp, P, P, i32, P, i32, i32, i32, P, P, P, P]
        L.or_forward_f32_full.restype = i32
        L.or_forward_emu_full.argtypes = [cfgp, P, P, i32, P, i32, i32, i32, P, P, P, P, i32]
        L.or_forward_emu_full.restype = i32
        L.or_emu_gemm.argtypes = [i32, P, P, P, i32, i32, i32, P, P, f32, P, P, P]
        L.or_emu_attention.argtypes = [P, P, i32, i32, i32]
        L.or_attention_f32.argtypes = [P, P, i32, i32, i32]
        L.or_emu_embed.argtypes = [P, P, P, i32, i32, f32, P]
        L.or_emu_norm_add.argtypes = [P, P, P, i32, i32, f32, P, P]
        L.or_emu_score.argtypes = [P, P, f32, P, i32, i32, P]
        L.or_row_stats.argtypes = [P, i32, i32, P]
        L.or_fold_layernorm.argtypes = [P, P, i32, i32, P, P]
        L.or_fold_layernorm_bias.argtypes = [P, P, P, P, i32, i32, P, P, P]
        L.or_rope_table.argtypes = [f32, i32, P]
        L.or_ref_permute_rope_rows.argtypes = [i32, P]
        L.or_ref_interleave_geglu_rows.argtypes = [i32, P]
        L.or_ref_phase_cost.argtypes = [i32] * 7
        L.or_ref_phase_cost.restype = ctypes.c_double
        L.or_ref_gemm_plan.argtypes = [i32] * 5 + [P, P]
        L.or_gelu.argtypes = [f32]
        L.or_gelu.restype = f32
        L.or_num_threads.restype = i32
        L.or_set_num_threads.argtypes = [i32]
        L.or_set_num_threads.restype = None
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def raw_size(c: Config) -> int:
    return lib().or_raw_size(ctypes.byref(c))


def init_random(c: Config, seed: int) -> np.ndarray:
    raw = np.empty(raw_size(c), np.float32)
    lib().or_init_random(ctypes.byref(c), seed, _p(raw))
    return raw


def normal(shape, seed: int, mean=0.0, std=1.0) -> np.ndarray:
    a = np.empty(shape, np.float32)
    lib().or_fill_normal(_p(a), a.size, seed, mean, std)
    return a


def forward_f32(c: Config, raw, ids, markers, qtype=0, trace=False, head_rows=0):
    """head_rows > 0: the head on the first head_rows rows only (or_forward_f32_head)."""
    ids = np.ascontiguousarray(ids, np.uint32)
    markers = np.ascontiguousarray(markers, np.uint32)
    logits = np.zeros(max(len(markers), 1), np.float32)
    tr = np.zeros((c.n_layers, len(ids), c.d_model), np.float32) if trace else None
    rc = lib().or_forward_f32_head(ctypes.byref(c), _p(raw), _p(ids), len(ids), _p(markers),
                                   len(markers), qtype, head_rows, _p(logits), _p(tr))
    if rc:
        raise ValueError("oracle: bad forward arguments")
    return (logits[:len(markers)], tr) if trace else logits[:len(markers)]


def forward_traced(c: Config, raw, ids, markers, qtype=0, head_rows=0, emulate=False, bugs=0):
    """The f32 model (or, emulate=True, the f16 emulation) with every stage traced:
    (logits, encoder stream [n_layers][n][D], head stream [n_head_layers + 1][nh][D] (its input,
    then after each head layer), scorer hidden layer after GELU [n_markers][scorer_hidden])."""
    ids = np.ascontiguousarray(ids, np.uint32)
    markers = np.ascontiguousarray(markers, np.uint32)
    n = len(ids)
    nh = head_rows if 0 < head_rows < n else n
    logits = np.zeros(max(len(markers), 1), np.float32)
    tr = np.zeros((c.n_layers, n, c.d_model), np.float32)
    ht = np.zeros((c.n_head_layers + 1, nh, c.d_model), np.float32)
    st = np.zeros((max(len(markers), 1), c.scorer_hidden), np.float32)
    if emulate:
        rc = lib().or_forward_emu_full(ctypes.byref(c), _p(raw), _p(ids), n, _p(markers),
                                       len(markers), qtype, head_rows, _p(logits), _p(tr), _p(ht),
                                       _p(st), bugs)
    else:
        rc = lib().or_forward_f32_full(ctypes.byref(c), _p(raw), _p(ids), n, _p(markers),
                                       len(markers), qtype, head_rows, _p(logits), _p(tr), _p(ht),
                                       _p(st))
    if rc:
        raise ValueError("oracle: bad forward arguments")
    k = len(markers)
    return logits[:k], tr, ht, st[:k]


def forward_emu(c: Config, raw, ids, markers, qtype=0, trace=False, bugs=0, head_rows=0):
    ids = np.ascontiguousarray(ids, np.uint32)
    markers = np.ascontiguousarray(markers, np.uint32)
    logits = np.zeros(max(len(markers), 1), np.float32)
    tr = np.zeros((c.n_layers, len(ids), c.d_model), np.float32) if trace else None
    rc = lib().or_forward_emu_head(ctypes.byref(c), _p(raw), _p(ids), len(ids), _p(markers),
                                   len(markers), qtype, head_rows, _p(logits), _p(tr), bugs)
    if rc:
        raise ValueError("oracle: bad forward arguments")
    return (logits[:len(markers)], tr) if trace else logits[:len(markers)]


def f16(a) -> np.ndarray:
    """f32 -> f16 bit patterns (round to nearest even)."""
    return np.ascontiguousarray(np.asarray(a, np.float32).astype(np.float16)).view(np.uint16)


def f32(h) -> np.ndarray:
    return np.asarray(h).view(np.float16).astype(np.float32)


def emu_gemm(epi, a16, w16, m, n, k, c16=None, stats_in=None, colsum=None, eps=1e-5, rope=None,
             bias=None, stats_out=None):
    """c = epilogue(a . w^T) as the kernels compute it (logical layouts); returns (c16, stats)."""
    n_out = n // 2 if epi & OR_GEGLU else n
    c = np.zeros((m, n_out), np.uint16) if c16 is None else np.ascontiguousarray(c16.copy())
    so = None
    if epi & OR_STATS:
        so = np.zeros(2 * m, np.float32) if stats_out is None else stats_out.copy()
    lib().or_emu_gemm(epi, _p(a16), _p(w16), _p(c), m, n, k, _p(stats_in), _p(colsum), eps,
                      _p(rope), _p(bias), _p(so))
    return c, so


def emu_attention(qkv16, n, heads, window):
    o = np.zeros((n, heads * 64), np.uint16)
    lib().or_emu_attention(_p(np.ascontiguousarray(qkv16)), _p(o), n, heads, window)
    return o


def attention_f32(qkv, n, heads, window):
    o = np.zeros((n, heads * 64), np.float32)
    lib().or_attention_f32(_p(np.ascontiguousarray(qkv, np.float32)), _p(o), n, heads, window)
    return o


def emu_embed(table16, gamma, ids, d, eps):
    ids = np.ascontiguousarray(ids, np.uint32)
    x = np.zeros((len(ids), d), np.uint16)
    lib().or_emu_embed(_p(table16), _p(gamma), _p(ids), len(ids), d, eps, _p(x))
    return x


def emu_norm_add(x16, gamma, add, eps):
    n, d = x16.shape
    out = np.zeros((n, d), np.uint16)
    st = np.zeros(2 * n, np.float32)
    lib().or_emu_norm_add(_p(x16), _p(gamma), _p(add), n, d, eps, _p(out), _p(st))
    return out, st


def emu_score(y16, w16, b, markers):
    markers = np.ascontiguousarray(markers, np.uint32)
    d = y16.shape[1]
    out = np.zeros(len(markers), np.float32)
    lib().or_emu_score(_p(y16), _p(w16), b, _p(markers), len(markers), d, _p(out))
    return out


def row_stats(x16):
    n, d = x16.shape
    st = np.zeros(2 * n, np.float32)
    lib().or_row_stats(_p(np.ascontiguousarray(x16)), n, d, _p(st))
    return st


def fold_layernorm(w, gamma):
    out, k = w.shape
    w16 = np.zeros((out, k), np.uint16)
    cs = np.zeros(out, np.float32)
    lib().or_fold_layernorm(_p(np.ascontiguousarray(w, np.float32)),
                            _p(np.ascontiguousarray(gamma, np.float32)), out, k, _p(w16), _p(cs))
    return w16, cs


def fold_layernorm_bias(w, gamma, beta, b):
    out, k = w.shape
    w16 = np.zeros((out, k), np.uint16)
    cs = np.zeros(out, np.float32)
    bias = np.zeros(out, np.float32)
    f = lambda a: _p(np.ascontiguousarray(a, np.float32))
    lib().or_fold_layernorm_bias(f(w), f(gamma), f(beta), f(b), out, k, _p(w16), _p(cs), _p(bias))
    return w16, cs, bias


def rope_table(theta, n):
    t = np.zeros((n, 32, 2), np.float32)
    lib().or_rope_table(theta, n, _p(t))
    return t


def ref_permute_rope_rows(n):
    r = np.zeros(n, np.int32)
    lib().or_ref_permute_rope_rows(n, _p(r))
    return r


def ref_interleave_geglu_rows(n):
    r = np.zeros(n, np.int32)
    lib().or_ref_interleave_geglu_rows(n, _p(r))
    return r


def ref_gemm_plan(n, cols, k, sms, per_sm):
    bm, z = ctypes.c_int(), ctypes.c_int()
    lib().or_ref_gemm_plan(n, cols, k, sms, per_sm, ctypes.byref(bm), ctypes.byref(z))
    return bm.value, z.value


def gelu(x: float) -> float:
    return lib().or_gelu(x)


def num_threads() -> int:
    return lib().or_num_threads()


def set_num_threads(n: int) -> None:
    lib().or_set_num_threads(n)
