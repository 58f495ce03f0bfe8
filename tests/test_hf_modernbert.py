"""The oracle's f32 encoder against Hugging Face transformers' ModernBertModel: an implementation of
the same architecture written outside this project (embedding LayerNorm; pre-norm layers without
biases, the first without an attention norm; global attention every third layer with RoPE theta
160000, +-64 sliding windows with theta 10000; a GeGLU MLP; the final norm), whose default
configuration is BASELINE config 0's encoder. Both run the same random weights, written by
julia_cuda_save_checkpoint under ModernBERT's tensor names and loaded into the transformers model
by those names. The head and the scorer (julia-rs's modules, absent here) are checked the same way
against torch's own modules of the form this project reads them as. This pins the oracle (and
through the GPU tests, the engine) to implementations written outside this project. CPU only
(transformers' eager attention in f32)."""
import json
import os
import struct

import numpy as np
import pytest

torch = pytest.importorskip("torch")
transformers = pytest.importorskip("transformers")


def read_safetensors(path):
    """name -> f32 numpy array of an F32 safetensors file."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        data = f.read()
    out = {}
    for name, t in header.items():
        if name == "__metadata__":
            continue
        assert t["dtype"] == "F32"
        a, b = t["data_offsets"]
        out[name] = np.frombuffer(data[a:b], np.float32).reshape(t["shape"])
    return out


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def oracle_cfg(O, c):
    return O.Config(*[getattr(c, f) for f, _ in c._fields_])


@pytest.mark.parametrize("n,full", [(37, False), (300, False), (293, True)])
def test_oracle_encoder_matches_transformers_modernbert(jc, O, tmp_path, n, full):
    """A small model (hidden 256, 4 layers) at one and several key tiles, and BASELINE config 0's
    encoder itself (hidden 768, 12 heads, 22 layers, 293 tokens)."""
    c = (jc.default_config(max_positions=1024) if full else
         jc.default_config(d_model=256, inter=384, n_layers=4, vocab=1000, max_positions=512))
    raw = O.init_random(oracle_cfg(O, c), 11)
    jc.save_checkpoint(str(tmp_path), c, raw)
    tensors = read_safetensors(os.path.join(str(tmp_path), "model.safetensors"))
    prefix = next(k[: -len("embeddings.tok_embeddings.weight")] for k in tensors
                  if k.endswith("embeddings.tok_embeddings.weight"))

    from transformers import ModernBertConfig, ModernBertModel
    layer_types = ["full_attention" if l % c.global_every == 0 else "sliding_attention"
                   for l in range(c.n_layers)]
    hf_cfg = ModernBertConfig(
        vocab_size=c.vocab, hidden_size=c.d_model, intermediate_size=c.inter,
        num_hidden_layers=c.n_layers, num_attention_heads=c.n_heads, norm_eps=c.norm_eps,
        norm_bias=False, attention_bias=False, mlp_bias=False, hidden_activation="gelu",
        local_attention=2 * c.window, max_position_embeddings=c.max_positions,
        layer_types=layer_types, pad_token_id=0, bos_token_id=0, eos_token_id=0, cls_token_id=0,
        sep_token_id=0,
        rope_parameters={"full_attention": {"rope_type": "default", "rope_theta": c.theta_global},
                         "sliding_attention": {"rope_type": "default",
                                               "rope_theta": c.theta_local}})
    hf_cfg._attn_implementation = "eager"
    model = ModernBertModel(hf_cfg).eval()
    state = {k[len(prefix):]: torch.from_numpy(v.copy()) for k, v in tensors.items()
             if k.startswith(prefix) and not k.startswith("head.") and not k.startswith("scorer.")
             and k != "type_emb.weight"}
    missing, unexpected = model.load_state_dict(state, strict=False)
    assert not missing and not unexpected, (missing, unexpected)

    rng = np.random.default_rng(n)
    ids = rng.integers(1, c.vocab, n).astype(np.uint32)
    with torch.no_grad():
        out = model(input_ids=torch.from_numpy(ids.astype(np.int64))[None],
                    output_hidden_states=True)
    hs = [h[0].numpy() for h in out.hidden_states]
    last = out.last_hidden_state[0].numpy()

    # transformers' hidden states: the embeddings, the input of every layer after the first, and
    # (in place of the last layer's output) the final norm of it.
    assert len(hs) == c.n_layers + 1
    qtype = 1
    _, tr, ht, _ = O.forward_traced(oracle_cfg(O, c), raw, ids, [0], qtype)
    worst = 0.0
    for l in range(c.n_layers - 1):
        e = rel_err(tr[l], hs[l + 1])
        worst = max(worst, e)
        assert e < 1e-4, f"layer {l}: {e:.2e}"
    # The head's input is the final norm (of the last layer's output) plus the question type's
    # embedding.
    assert np.array_equal(hs[-1], last)
    e = rel_err(ht[0] - tensors["type_emb.weight"][qtype], last)
    assert e < 1e-4, f"final norm: {e:.2e}"
    print(f"n={n}: worst layer {worst:.2e}, final norm {e:.2e}")


def test_oracle_forward_matches_transformers_and_torch_modules(jc, O, tmp_path):
    """The whole f32 forward of BASELINE config 0 (293 tokens, 4 markers) against a forward built
    from independent implementations loaded with the same checkpoint: transformers' ModernBertModel
    for the encoder, the question type's embedding added to its final norm, two
    torch.nn.TransformerEncoderLayer (pre-norm, ReLU; the head's tensor names are theirs) over
    every row, and the scorer as torch.nn.LayerNorm, Linear, GELU, Linear on the marker rows. The
    head's stream after each layer and the logits must agree."""
    from transformers import ModernBertConfig, ModernBertModel
    c = jc.default_config(max_positions=1024)
    raw = O.init_random(oracle_cfg(O, c), 23)
    jc.save_checkpoint(str(tmp_path), c, raw)
    tensors = read_safetensors(os.path.join(str(tmp_path), "model.safetensors"))
    prefix = next(k[: -len("embeddings.tok_embeddings.weight")] for k in tensors
                  if k.endswith("embeddings.tok_embeddings.weight"))
    layer_types = ["full_attention" if l % c.global_every == 0 else "sliding_attention"
                   for l in range(c.n_layers)]
    hf_cfg = ModernBertConfig(
        vocab_size=c.vocab, hidden_size=c.d_model, intermediate_size=c.inter,
        num_hidden_layers=c.n_layers, num_attention_heads=c.n_heads, norm_eps=c.norm_eps,
        norm_bias=False, attention_bias=False, mlp_bias=False, hidden_activation="gelu",
        local_attention=2 * c.window, max_position_embeddings=c.max_positions,
        layer_types=layer_types, pad_token_id=0, bos_token_id=0, eos_token_id=0, cls_token_id=0,
        sep_token_id=0,
        rope_parameters={"full_attention": {"rope_type": "default", "rope_theta": c.theta_global},
                         "sliding_attention": {"rope_type": "default",
                                               "rope_theta": c.theta_local}})
    hf_cfg._attn_implementation = "eager"
    enc = ModernBertModel(hf_cfg).eval()
    t = lambda a: torch.from_numpy(np.array(a))  # noqa: E731
    missing, unexpected = enc.load_state_dict(
        {k[len(prefix):]: t(v) for k, v in tensors.items() if k.startswith(prefix)
         and not k.startswith(("head.", "scorer.")) and k != "type_emb.weight"}, strict=False)
    assert not missing and not unexpected
    head = torch.nn.ModuleList([
        torch.nn.TransformerEncoderLayer(c.d_model, c.n_heads, dim_feedforward=c.head_ff,
                                         dropout=0.0, activation="relu", layer_norm_eps=c.head_eps,
                                         batch_first=True, norm_first=True)
        for _ in range(c.n_head_layers)]).eval()
    head.load_state_dict({k[len("head.layers."):]: t(v) for k, v in tensors.items()
                          if k.startswith("head.layers.")}, strict=True)
    norm = torch.nn.LayerNorm(c.d_model, eps=c.head_eps)
    lin1 = torch.nn.Linear(c.d_model, c.scorer_hidden)
    lin2 = torch.nn.Linear(c.scorer_hidden, 1)
    for mod, name in ((norm, "scorer.norm"), (lin1, "scorer.lin1"), (lin2, "scorer.lin2")):
        mod.load_state_dict({"weight": t(tensors[name + ".weight"]),
                             "bias": t(tensors[name + ".bias"])})

    rng = np.random.default_rng(293)
    n, qtype = 293, 2
    ids = rng.integers(1, c.vocab, n).astype(np.uint32)
    markers = np.sort(rng.choice(n, 4, replace=False)).astype(np.uint32)
    with torch.no_grad():
        x = enc(input_ids=t(ids.astype(np.int64))[None]).last_hidden_state
        x = x + t(tensors["type_emb.weight"][qtype])
        stream = [x[0].numpy()]
        for layer in head:
            x = layer(x)
            stream.append(x[0].numpy())
        z = x[0, t(markers.astype(np.int64))]
        want = lin2(torch.nn.functional.gelu(lin1(norm(z))))[:, 0].numpy()

    logits, _, ht, _ = O.forward_traced(oracle_cfg(O, c), raw, ids, markers, qtype)
    for s in range(c.n_head_layers + 1):
        e = rel_err(ht[s], stream[s])
        assert e < 2e-6, f"head stage {s}: {e:.2e}"
    d = np.max(np.abs(logits - want)) / max(float(np.sqrt(np.mean(want.astype(np.float64) ** 2))), 1e-30)
    assert d < 1e-4, (logits, want)
    print(f"logits {logits} vs {want}: max |d| / rms {d:.2e}")


def test_torch_runtime_matches_the_oracle(jc, O, tmp_path):
    """baseline/torch_runtime.py (the reference's torch-runtime comparison assembled from
    transformers' ModernBertModel and torch modules; what `bench.py --torch-runtime` runs on the
    GPU), in f32 on the CPU, against the oracle's f32 forward on a small model at one key tile and
    at several: the same logits."""
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "baseline"))
    from torch_runtime import TorchRuntime
    c = jc.default_config(d_model=256, inter=384, n_layers=4, vocab=1000, max_positions=512)
    raw = O.init_random(oracle_cfg(O, c), 5)
    jc.save_checkpoint(str(tmp_path), c, raw)
    rt = TorchRuntime(str(tmp_path), device="cpu", dtype="fp32", attn="eager")
    rng = np.random.default_rng(7)
    for n, qtype in ((37, 0), (300, 2)):
        ids = rng.integers(0, c.vocab, n).astype(np.uint32)
        markers = np.sort(rng.choice(n, 4, replace=False)).astype(np.uint32)
        got = rt.forward(ids, markers, qtype)
        want = np.asarray(O.forward_f32(oracle_cfg(O, c), raw, ids, markers, qtype), np.float64)
        rms = max(float(np.sqrt(np.mean(want ** 2))), 1e-30)
        d = float(np.max(np.abs(got - want))) / rms
        assert d < 1e-4, (n, got, want)


def test_torch_runtime_serves_request_jsonl(jc, O, tmp_path, monkeypatch, capsys):
    """baseline/torch_runtime.py as a script: request JSONL in (the julia-cuda executable's
    format, question types by number or name), result lines out with the oracle's logits, their
    softmax and the argmax marker, as tools/score.py reads them."""
    import io
    import json as js
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "baseline"))
    import torch_runtime
    c = jc.default_config(d_model=256, inter=384, n_layers=4, vocab=1000, max_positions=512)
    raw = O.init_random(oracle_cfg(O, c), 9)
    jc.save_checkpoint(str(tmp_path), c, raw)
    rng = np.random.default_rng(3)
    reqs = []
    for n, q in ((50, "score"), (130, 2)):
        ids = rng.integers(0, c.vocab, n).astype(np.uint32)
        markers = np.sort(rng.choice(n, 3, replace=False)).astype(np.uint32)
        reqs.append((ids, markers, q))
    text = "".join(js.dumps({"ids": ids.tolist(), "markers": m.tolist(), "qtype": q}) + "\n"
                   for ids, m, q in reqs)
    monkeypatch.setattr(sys, "stdin", io.StringIO(text))
    assert torch_runtime.main([str(tmp_path), "--device", "cpu", "--dtype", "fp32",
                               "--attn", "eager"]) == 0
    lines = [js.loads(l) for l in capsys.readouterr().out.splitlines() if l.strip()]
    assert len(lines) == 2
    for (ids, m, q), res in zip(reqs, lines):
        want = np.asarray(O.forward_f32(oracle_cfg(O, c), raw, ids, m,
                                        torch_runtime.QTYPES.get(q, q)), np.float64)
        got = np.asarray(res["logits"])
        assert np.max(np.abs(got - want)) / max(float(np.sqrt(np.mean(want ** 2))), 1e-30) < 1e-4
        assert res["choice"] == int(np.argmax(got))
        assert abs(sum(res["probabilities"]) - 1.0) < 1e-9 and res["truncated"] is False
