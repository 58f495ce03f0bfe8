"""An independent torch-CPU f32 restatement of the Julia-1 forward pass, used to pin the C oracle.

Written from the same semantics (the reference's src/check.rs:177-224 `trace` and :484-548
`head_trace`: pre-LayerNorm ModernBERT encoder with rotate-half RoPE, global / +-64-window
attention and GeGLU; final norm + type embedding; two pre-LN nn.TransformerEncoderLayer head
layers with ReLU; LayerNorm -> lin1 -> GELU -> lin2 scorer on the marker rows), but with torch
primitives and its own reading of the raw format, so a mistake in one is unlikely to be in both.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F


def raw_tensors(c, raw: np.ndarray) -> dict:
    """Splits the raw f32 buffer into named tensors (order documented in include/julia_cuda.h)."""
    D, I, FF, S, V = c.d_model, c.inter, c.head_ff, c.scorer_hidden, c.vocab
    t = torch.from_numpy(np.asarray(raw, np.float32))
    at = 0
    out = {}

    def take(name, *shape):
        nonlocal at
        n = int(np.prod(shape)) if shape else 0
        out[name] = t[at:at + n].reshape(*shape) if n else None
        at += n

    take("tok", V, D)
    take("emb_norm", D)
    for l in range(c.n_layers):
        if l == 0:
            out[f"attn_norm{l}"] = None
        else:
            take(f"attn_norm{l}", D)
        take(f"wqkv{l}", 3 * D, D)
        take(f"wo{l}", D, D)
        take(f"mlp_norm{l}", D)
        take(f"wi{l}", 2 * I, D)
        take(f"wo_mlp{l}", D, I)
    take("final_norm", D)
    take("type_emb", c.n_qtypes, D)
    for l in range(c.n_head_layers):
        take(f"n1w{l}", D)
        take(f"n1b{l}", D)
        take(f"inw{l}", 3 * D, D)
        take(f"inb{l}", 3 * D)
        take(f"outw{l}", D, D)
        take(f"outb{l}", D)
        take(f"n2w{l}", D)
        take(f"n2b{l}", D)
        take(f"l1w{l}", FF, D)
        take(f"l1b{l}", FF)
        take(f"l2w{l}", D, FF)
        take(f"l2b{l}", D)
    take("snw", D)
    take("snb", D)
    take("s1w", S, D)
    take("s1b", S)
    take("s2w", 1, S)
    take("s2b", 1)
    assert at == t.numel(), (at, t.numel())
    return out


def ln64(x, w, b, eps):
    """LayerNorm with f64 statistics, f32 result (src/check.rs:227-242)."""
    x64 = x.double()
    mean = x64.mean(-1, keepdim=True)
    var = ((x64 - mean) ** 2).mean(-1, keepdim=True)
    y = (x64 - mean) / torch.sqrt(var + eps) * w.double()
    if b is not None:
        y = y + b.double()
    return y.float()


def gelu_as(x):
    """GELU with the Abramowitz & Stegun 7.1.26 erf (the kernels' and julia-rs's formula)."""
    x64 = x.double()
    t = 1.0 / (1.0 + 0.2316419 * x64.abs())
    p = ((((1.061405429 * t - 1.453152027) * t + 1.421413741) * t - 0.284496736) * t
         + 0.254829592) * t
    q = 0.5 * p * torch.exp(-x64 * x64 / 2)
    return (x64 * torch.where(x64 >= 0, 1 - q, q)).float()


def rope_cos_sin(theta: float, n: int):
    j = torch.arange(32, dtype=torch.float32)
    inv = 1.0 / torch.pow(torch.tensor(theta, dtype=torch.float32), 2 * j / 64.0)
    ang = torch.arange(n, dtype=torch.float32)[:, None] * inv[None, :]
    return torch.cos(ang), torch.sin(ang)


def rope(x, cos, sin, heads):
    """Rotate-half on dims (i, i + 32) of each 64-wide head; x [n, heads*64]."""
    n = x.shape[0]
    h = x.view(n, heads, 64)
    x1, x2 = h[..., :32], h[..., 32:]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1).reshape(n, heads * 64)


def attention(q, k, v, heads, window):
    n = q.shape[0]
    qh = q.view(n, heads, 64).transpose(0, 1)
    kh = k.view(n, heads, 64).transpose(0, 1)
    vh = v.view(n, heads, 64).transpose(0, 1)
    s = qh @ kh.transpose(1, 2) / 8.0
    if window > 0:
        i = torch.arange(n)
        far = (i[:, None] - i[None, :]).abs() > window
        s = s.masked_fill(far[None], float("-inf"))
    p = torch.softmax(s, -1)
    return (p @ vh).transpose(0, 1).reshape(n, heads * 64)


def forward(c, raw, ids, markers, qtype=0, trace=False, head_rows=0):
    """head_rows > 0: the head (final norm, head layers, marker rows) sees only the first
    head_rows rows of the encoder's output."""
    W = raw_tensors(c, raw)
    D, H, I = c.d_model, c.n_heads, c.inter
    n = len(ids)
    ids_t = torch.as_tensor(np.asarray(ids, np.int64))
    cg, sg = rope_cos_sin(c.theta_global, n)
    cl, sl = rope_cos_sin(c.theta_local, n)
    x = ln64(W["tok"][ids_t], W["emb_norm"], None, c.norm_eps)
    tr = []
    for l in range(c.n_layers):
        glob = l % c.global_every == 0
        h = x if W[f"attn_norm{l}"] is None else ln64(x, W[f"attn_norm{l}"], None, c.norm_eps)
        qkv = h @ W[f"wqkv{l}"].T
        q, k, v = qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:]
        cs, sn = (cg, sg) if glob else (cl, sl)
        q, k = rope(q, cs, sn, H), rope(k, cs, sn, H)
        o = attention(q, k, v, H, 0 if glob else c.window)
        x = x + o @ W[f"wo{l}"].T
        h = ln64(x, W[f"mlp_norm{l}"], None, c.norm_eps)
        hh = h @ W[f"wi{l}"].T
        m = gelu_as(hh[:, :I]) * hh[:, I:]
        x = x + m @ W[f"wo_mlp{l}"].T
        tr.append(x.clone())
    if 0 < head_rows < n:
        x = x[:head_rows]
    x = ln64(x, W["final_norm"], None, c.norm_eps) + W["type_emb"][qtype]
    for l in range(c.n_head_layers):
        h = ln64(x, W[f"n1w{l}"], W[f"n1b{l}"], c.head_eps)
        qkv = h @ W[f"inw{l}"].T + W[f"inb{l}"]
        o = attention(qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:], H, 0)
        x = x + o @ W[f"outw{l}"].T + W[f"outb{l}"]
        h = ln64(x, W[f"n2w{l}"], W[f"n2b{l}"], c.head_eps)
        f = torch.relu(h @ W[f"l1w{l}"].T + W[f"l1b{l}"])
        x = x + f @ W[f"l2w{l}"].T + W[f"l2b{l}"]
    z = x[torch.as_tensor(np.asarray(markers, np.int64))]
    z = ln64(z, W["snw"], W["snb"], c.head_eps)
    y = gelu_as(z @ W["s1w"].T + W["s1b"])
    logits = (y @ W["s2w"].T + W["s2b"])[:, 0]
    if trace:
        return logits.numpy(), torch.stack(tr).numpy()
    return logits.numpy()
