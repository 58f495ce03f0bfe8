"""Checkpoint directories in the reference's layout (src/checkpoint.rs:27-62): model.safetensors +
encoder/config.json + julia_config.json, read by julia_cuda_read_checkpoint into the raw format
and prepared (julia_cuda_prepare_host) into the arenas an engine uploads. The safetensors files
here are written by an independent writer (numpy + json, below), not by the library, so the
reader is checked against the format itself. CPU only, except the last test (the engine loaded
from such a directory on the GPU)."""
import json
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")


def small_cfg(jc):
    return jc.default_config(d_model=128, inter=128, n_layers=3, vocab=300, head_ff=256,
                             scorer_hidden=64, max_positions=256, n_head_layers=2)


def tensor_table(jc, cfg, raw, prefix="model."):
    """(name, shape, values) of every raw tensor under the documented default names, in raw order
    (julia_cuda.h: the raw format's order)."""
    D, I, F, S = cfg.d_model, cfg.inter, cfg.head_ff, cfg.scorer_hidden
    off = list(jc.raw_offsets(cfg)) + [raw.size]
    spec = [("embeddings.tok_embeddings.weight", (cfg.vocab, D), True),
            ("embeddings.norm.weight", (D,), True)]
    for l in range(cfg.n_layers):
        p = f"layers.{l}."
        spec += [(p + "attn_norm.weight", (D,) if l else (0,), True),
                 (p + "attn.Wqkv.weight", (3 * D, D), True), (p + "attn.Wo.weight", (D, D), True),
                 (p + "mlp_norm.weight", (D,), True), (p + "mlp.Wi.weight", (2 * I, D), True),
                 (p + "mlp.Wo.weight", (D, I), True)]
    spec += [("final_norm.weight", (D,), True), ("type_emb.weight", (cfg.n_qtypes, D), False)]
    for l in range(cfg.n_head_layers):
        p = f"head.layers.{l}."
        spec += [(p + "norm1.weight", (D,), False), (p + "norm1.bias", (D,), False),
                 (p + "self_attn.in_proj_weight", (3 * D, D), False),
                 (p + "self_attn.in_proj_bias", (3 * D,), False),
                 (p + "self_attn.out_proj.weight", (D, D), False),
                 (p + "self_attn.out_proj.bias", (D,), False), (p + "norm2.weight", (D,), False),
                 (p + "norm2.bias", (D,), False), (p + "linear1.weight", (F, D), False),
                 (p + "linear1.bias", (F,), False), (p + "linear2.weight", (D, F), False),
                 (p + "linear2.bias", (D,), False)]
    spec += [("scorer.norm.weight", (D,), False), ("scorer.norm.bias", (D,), False),
             ("scorer.lin1.weight", (S, D), False), ("scorer.lin1.bias", (S,), False),
             ("scorer.lin2.weight", (1, S), False), ("scorer.lin2.bias", (1,), False)]
    assert len(spec) == len(off) - 1
    out = []
    for i, (name, shape, enc) in enumerate(spec):
        v = raw[off[i]:off[i + 1]]
        assert v.size == int(np.prod(shape))
        if v.size:
            out.append(((prefix if enc else "") + name, shape, v.reshape(shape)))
    return out


def write_safetensors(path, tensors, dtype="F32", extra_meta=True):
    """The safetensors format from its specification: an 8-byte little-endian header length, a
    JSON header {name: {dtype, shape, data_offsets}}, the data section."""
    np_dt = {"F32": np.float32, "F16": np.float16}
    header, blobs, at = {}, [], 0
    if extra_meta:
        header["__metadata__"] = {"format": "pt"}
    for name, shape, v in tensors:
        if dtype == "BF16":
            b = (np.ascontiguousarray(v, np.float32).view(np.uint32) >> 16).astype(np.uint16).tobytes()
        else:
            b = np.ascontiguousarray(v, np_dt[dtype]).tobytes()
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [at, at + len(b)]}
        blobs.append(b)
        at += len(b)
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(len(h).to_bytes(8, "little"))
        f.write(h)
        for b in blobs:
            f.write(b)


def write_dir(jc, d, cfg, raw, prefix="model.", dtype="F32", julia_config=True, rename=None):
    os.makedirs(os.path.join(d, "encoder"), exist_ok=True)
    table = tensor_table(jc, cfg, raw, prefix)
    if rename:
        table = [(rename.get(n, n), s, v) for n, s, v in table]
    write_safetensors(os.path.join(d, "model.safetensors"), table, dtype)
    with open(os.path.join(d, "encoder", "config.json"), "w") as f:
        json.dump({"model_type": "modernbert", "hidden_size": cfg.d_model,
                   "intermediate_size": cfg.inter, "num_hidden_layers": cfg.n_layers,
                   "num_attention_heads": cfg.n_heads, "vocab_size": cfg.vocab,
                   "norm_eps": cfg.norm_eps, "local_attention": 2 * cfg.window,
                   "global_attn_every_n_layers": cfg.global_every,
                   "max_position_embeddings": cfg.max_positions,
                   "global_rope_theta": cfg.theta_global, "local_rope_theta": cfg.theta_local}, f)
    if julia_config:
        with open(os.path.join(d, "julia_config.json"), "w") as f:
            json.dump({"head_layers": cfg.n_head_layers, "head_ff": cfg.head_ff,
                       "scorer_hidden": cfg.scorer_hidden, "n_qtypes": cfg.n_qtypes,
                       "head_eps": cfg.head_eps}, f)


def cfg_tuple(c):
    return tuple(getattr(c, f) for f, _ in c._fields_)


@pytest.mark.parametrize("prefix", ["model.", "encoder.", ""])
def test_checkpoint_reads_bit_for_bit_and_prepares_the_same_arenas(jc, tmp_path, prefix):
    cfg = small_cfg(jc)
    raw = jc.init_random(cfg, 5)
    write_dir(jc, str(tmp_path), cfg, raw, prefix=prefix)
    got_cfg, got = jc.read_checkpoint(str(tmp_path))
    assert cfg_tuple(got_cfg) == cfg_tuple(cfg)
    assert got.view(np.uint32).tobytes() == raw.view(np.uint32).tobytes()
    a16, a32 = jc.prepare_host(cfg, raw, 256)
    b16, b32 = jc.prepare_host(got_cfg, got, 256)
    assert np.array_equal(a16, b16) and a32.view(np.uint32).tobytes() == b32.view(np.uint32).tobytes()


def test_widths_come_from_the_shapes_without_julia_config(jc, tmp_path):
    cfg = small_cfg(jc).replace(head_ff=192, scorer_hidden=128, n_qtypes=5)
    raw = jc.init_random(cfg, 6)
    write_dir(jc, str(tmp_path), cfg, raw, julia_config=False)
    got_cfg, got = jc.read_checkpoint(str(tmp_path))
    assert (got_cfg.head_ff, got_cfg.scorer_hidden, got_cfg.n_qtypes, got_cfg.n_head_layers) == \
        (192, 128, 5, 2)
    assert np.array_equal(got, raw)


@pytest.mark.parametrize("dtype", ["F16", "BF16"])
def test_half_precision_tensors(jc, tmp_path, dtype):
    cfg = small_cfg(jc)
    raw = jc.init_random(cfg, 7)
    write_dir(jc, str(tmp_path), cfg, raw, dtype=dtype)
    _, got = jc.read_checkpoint(str(tmp_path))
    if dtype == "F16":
        want = raw.astype(np.float16).astype(np.float32)
    else:  # truncation, as the writer above stores it
        want = ((raw.view(np.uint32) >> 16) << 16).view(np.float32)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("dtype", [0, 1, 2])
def test_library_writer_round_trip(jc, tmp_path, dtype):
    cfg = small_cfg(jc)
    raw = jc.init_random(cfg, 8)
    jc.save_checkpoint(str(tmp_path), cfg, raw, dtype)
    got_cfg, got = jc.read_checkpoint(str(tmp_path))
    assert cfg_tuple(got_cfg) == cfg_tuple(cfg)
    if dtype == 0:
        assert np.array_equal(got, raw)
    elif dtype == 1:
        assert np.array_equal(got, raw.astype(np.float16).astype(np.float32))
    else:  # round to nearest even
        u = raw.view(np.uint32).astype(np.uint64)
        r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16 << 16).astype(np.uint32)
        assert np.array_equal(got, r.view(np.float32))


def test_name_overrides(jc, tmp_path):
    """Head / scorer names live in julia-rs (absent): jc_names.json maps the documented names to
    a file's own."""
    cfg = small_cfg(jc)
    raw = jc.init_random(cfg, 9)
    rename = {"scorer.lin1.weight": "classifier.dense.weight", "type_emb.weight": "qtype.weight",
              "model.final_norm.weight": "model.norm_final.weight"}
    write_dir(jc, str(tmp_path), cfg, raw, rename=rename)
    with pytest.raises(jc.JuliaCudaError, match="no tensor"):
        jc.read_checkpoint(str(tmp_path))
    with open(tmp_path / "jc_names.json", "w") as f:
        json.dump({"names": {"scorer.lin1.weight": "classifier.dense.weight",
                             "type_emb.weight": "qtype.weight",
                             "final_norm.weight": "model.norm_final.weight"}}, f)
    _, got = jc.read_checkpoint(str(tmp_path))
    assert np.array_equal(got, raw)


def test_bad_checkpoints_are_rejected(jc, tmp_path):
    cfg = small_cfg(jc)
    raw = jc.init_random(cfg, 10)
    d = str(tmp_path)
    with pytest.raises(jc.JuliaCudaError, match="cannot read"):
        jc.read_checkpoint(d)
    # a shape that disagrees with the config
    write_dir(jc, d, cfg, raw)
    with open(os.path.join(d, "encoder", "config.json")) as f:
        enc = json.load(f)
    enc["intermediate_size"] = 192
    with open(os.path.join(d, "encoder", "config.json"), "w") as f:
        json.dump(enc, f)
    with pytest.raises(jc.JuliaCudaError, match="shape"):
        jc.read_checkpoint(d)
    # an unsupported dtype
    write_dir(jc, d, cfg, raw)
    path = os.path.join(d, "model.safetensors")
    with open(path, "rb") as f:
        blob = f.read()
    n = int.from_bytes(blob[:8], "little")
    header = json.loads(blob[8:8 + n])
    header["scorer.lin2.bias"]["dtype"] = "I32"
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(len(h).to_bytes(8, "little") + h + blob[8 + n:])
    with pytest.raises(jc.JuliaCudaError, match="dtype"):
        jc.read_checkpoint(d)
    # a truncated file: the header's offsets reach past the data
    write_dir(jc, d, cfg, raw)
    with open(path, "rb") as f:
        blob = f.read()
    with open(path, "wb") as f:
        f.write(blob[:len(blob) - 100])
    with pytest.raises(jc.JuliaCudaError, match="outside the data section"):
        jc.read_checkpoint(d)
    # a header that is not JSON
    with open(path, "wb") as f:
        f.write((5).to_bytes(8, "little") + b"{nope")
    with pytest.raises(jc.JuliaCudaError, match="header"):
        jc.read_checkpoint(d)
    # a header length past the end of the file
    with open(path, "wb") as f:
        f.write((10 ** 9).to_bytes(8, "little") + b"{}")
    with pytest.raises(jc.JuliaCudaError, match="exceeds"):
        jc.read_checkpoint(d)


@pytest.mark.gpu
def test_engine_loads_a_checkpoint_directory(jc, O, tmp_path):
    """julia_cuda_load on a safetensors directory: the same logits, bit for bit, as the engine
    built from the same raw weights."""
    cfg = small_cfg(jc)
    raw = jc.init_random(cfg, 11)
    write_dir(jc, str(tmp_path), cfg, raw)
    a = jc.Engine.load(str(tmp_path), max_length=256)
    b = jc.Engine.load_raw(cfg, raw, max_length=256)
    try:
        req = [(np.arange(90, dtype=np.uint32) % cfg.vocab, np.array([0, 45, 89], np.uint32), 1)]
        la, _ = a.run(req)
        lb, _ = b.run(req)
        assert np.array_equal(la[0], lb[0])
        oc = O.Config(*cfg_tuple(cfg))
        assert np.max(np.abs(la[0] - O.forward_emu(oc, raw, *req[0]))) < 2e-3
    finally:
        a.close()
        b.close()
