"""The reference's torch-runtime comparison, assembled from implementations present here.

The reference measures the original Julia-1 runtime beside its own engine (tools/torch_baseline.py:
the PyTorch model from the Hugging Face snapshot, BF16 autocast by default, fp16 or fp32 on
request, one request at a time on the GPU, wall time per request) and compares the two runs'
answers with tools/score.py. That runtime and its snapshot are not available here, so this module
builds the same network from libraries written outside this project, loaded from a checkpoint
directory in the reference's layout (model.safetensors, encoder/config.json, julia_config.json; as
julia_cuda_save_checkpoint writes it, default tensor names):

  - the encoder: transformers' ModernBertModel (embedding LayerNorm, pre-norm layers without
    biases, global attention every `global_attn_every_n_layers` layers with `global_rope_theta`,
    sliding windows of `local_attention` tokens with `local_rope_theta`, GeGLU MLP, final norm);
  - the question type's embedding added to every row of the encoder's output;
  - the head: one torch.nn.TransformerEncoderLayer per head layer (pre-norm, ReLU), loaded by its
    own parameter names (`head.layers.<i>.*`);
  - the scorer on the marker rows: torch.nn.LayerNorm, Linear, GELU, Linear (`scorer.*`).

tests/test_hf_modernbert.py pins this assembly to the oracle's f32 forward on the CPU, and
`python bench.py --torch-runtime` runs it on a B200 beside this library (agreement and latency).
Run as a script it serves request JSONL like the julia-cuda executable (see main()).
"""
import json
import os
import struct

import numpy as np


def read_safetensors(path: str) -> dict:
    """name -> f32 numpy array, for the F32 / F16 / BF16 tensors of a safetensors file."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        data = f.read()
    out = {}
    for name, t in header.items():
        if name == "__metadata__":
            continue
        a, b = t["data_offsets"]
        raw = data[a:b]
        if t["dtype"] == "F32":
            v = np.frombuffer(raw, np.float32)
        elif t["dtype"] == "F16":
            v = np.frombuffer(raw, np.float16).astype(np.float32)
        elif t["dtype"] == "BF16":
            v = (np.frombuffer(raw, np.uint16).astype(np.uint32) << 16).view(np.float32)
        else:
            raise ValueError(f"{name}: dtype {t['dtype']} (F32, F16 or BF16 only)")
        out[name] = v.reshape(t["shape"])
    return out


class TorchRuntime:
    """The assembled model on one device. dtype: "bf16" / "fp16" run under torch.autocast (the
    reference runtime's default is BF16), "fp32" without it; attn: transformers' attention
    implementation for the encoder ("sdpa" or "eager")."""

    def __init__(self, model_dir: str, device: str = "cuda", dtype: str = "bf16",
                 attn: str = "sdpa"):
        import torch
        from transformers import ModernBertConfig, ModernBertModel

        self.torch = torch
        self.device = torch.device(device)
        self.autocast = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": None}[dtype]
        with open(os.path.join(model_dir, "encoder", "config.json")) as f:
            enc = json.load(f)
        with open(os.path.join(model_dir, "julia_config.json")) as f:
            jul = json.load(f)
        tensors = read_safetensors(os.path.join(model_dir, "model.safetensors"))
        tail = "embeddings.tok_embeddings.weight"
        prefix = next(k[: -len(tail)] for k in tensors if k.endswith(tail))

        layers, every = enc["num_hidden_layers"], enc.get("global_attn_every_n_layers", 3)
        d, heads = enc["hidden_size"], enc.get("num_attention_heads", enc["hidden_size"] // 64)
        hf = ModernBertConfig(
            vocab_size=enc["vocab_size"], hidden_size=d, intermediate_size=enc["intermediate_size"],
            num_hidden_layers=layers, num_attention_heads=heads,
            norm_eps=enc.get("norm_eps", 1e-5), norm_bias=False, attention_bias=False,
            mlp_bias=False, hidden_activation="gelu",
            local_attention=enc.get("local_attention", 128),
            max_position_embeddings=enc.get("max_position_embeddings", 8192),
            layer_types=["full_attention" if l % every == 0 else "sliding_attention"
                         for l in range(layers)],
            pad_token_id=0, bos_token_id=0, eos_token_id=0, cls_token_id=0, sep_token_id=0,
            rope_parameters={
                "full_attention": {"rope_type": "default",
                                   "rope_theta": enc.get("global_rope_theta", 160000.0)},
                "sliding_attention": {"rope_type": "default",
                                      "rope_theta": enc.get("local_rope_theta", 10000.0)}})
        hf._attn_implementation = attn
        t = lambda a: torch.from_numpy(np.array(a))  # noqa: E731
        self.encoder = ModernBertModel(hf)
        missing, unexpected = self.encoder.load_state_dict(
            {k[len(prefix):]: t(v) for k, v in tensors.items() if k.startswith(prefix)
             and not k.startswith(("head.", "scorer.")) and k != "type_emb.weight"}, strict=False)
        if missing or unexpected:
            raise ValueError(f"encoder tensors: missing {missing}, unexpected {unexpected}")
        n_head = jul.get("head_layers", 2)
        self.head = torch.nn.ModuleList([
            torch.nn.TransformerEncoderLayer(d, heads, dim_feedforward=jul["head_ff"], dropout=0.0,
                                             activation="relu", layer_norm_eps=jul["head_eps"],
                                             batch_first=True, norm_first=True)
            for _ in range(n_head)])
        self.head.load_state_dict({k[len("head.layers."):]: t(v) for k, v in tensors.items()
                                   if k.startswith("head.layers.")}, strict=True)
        self.norm = torch.nn.LayerNorm(d, eps=jul["head_eps"])
        self.lin1 = torch.nn.Linear(d, jul["scorer_hidden"])
        self.lin2 = torch.nn.Linear(jul["scorer_hidden"], 1)
        for mod, name in ((self.norm, "scorer.norm"), (self.lin1, "scorer.lin1"),
                          (self.lin2, "scorer.lin2")):
            mod.load_state_dict({"weight": t(tensors[name + ".weight"]),
                                 "bias": t(tensors[name + ".bias"])})
        self.type_emb = t(tensors["type_emb.weight"])
        for m in (self.encoder, self.head, self.norm, self.lin1, self.lin2):
            m.to(self.device).eval()
        self.type_emb = self.type_emb.to(self.device)

    def forward(self, ids, markers, qtype: int) -> np.ndarray:
        """One request (token ids, marker rows, question type): its logits, one per marker, on the
        host (the device round trip included, as the reference runtime returns them)."""
        torch = self.torch
        ids_t = torch.as_tensor(np.asarray(ids, np.int64)).to(self.device)[None]
        mk = torch.as_tensor(np.asarray(markers, np.int64)).to(self.device)
        with torch.inference_mode(), torch.autocast(self.device.type,
                                                    dtype=self.autocast or torch.float32,
                                                    enabled=self.autocast is not None):
            x = self.encoder(input_ids=ids_t).last_hidden_state
            x = x + self.type_emb[qtype]
            for layer in self.head:
                x = layer(x)
            z = x[0, mk]
            logits = self.lin2(torch.nn.functional.gelu(self.lin1(self.norm(z))))[:, 0]
        return logits.float().cpu().numpy()


QTYPES = {"choice": 0, "score": 1, "noul": 2}


def result_line(logits: np.ndarray, ms: float) -> dict:
    """A result in the format the julia-cuda executable writes (and tools/score.py reads): the
    marker logits, their softmax, the argmax marker, "truncated" false, and the wall time."""
    lg = np.asarray(logits, np.float64)
    p = np.exp(lg - lg.max()) if lg.size else lg
    return {"logits": [float(v) for v in lg],
            "probabilities": [float(v) for v in p / p.sum()] if lg.size else [],
            "choice": int(np.argmax(lg)) if lg.size else None, "truncated": False,
            "wall_ms": ms}


def main(argv=None) -> int:
    """python baseline/torch_runtime.py MODEL_DIR [--device cuda] [--dtype bf16] < requests.jsonl
    > results.jsonl: token-id requests ({"ids": [...], "markers": [...], "qtype": 0-2 or
    "choice" / "score" / "noul"}, as the julia-cuda executable reads them) one at a time through
    the torch runtime, one result line each; julia-cuda_b200/scoring.py compares two such runs."""
    import argparse
    import sys
    import time
    ap = argparse.ArgumentParser()
    ap.add_argument("model_dir")
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "fp16", "fp32"])
    ap.add_argument("--attn", default="sdpa", choices=["sdpa", "eager"])
    args = ap.parse_args(argv)
    rt = TorchRuntime(args.model_dir, device=args.device, dtype=args.dtype, attn=args.attn)
    for line in sys.stdin:
        if not line.strip():
            continue
        req = json.loads(line)
        q = req.get("qtype", 0)
        q = QTYPES[q] if isinstance(q, str) else int(q)
        t0 = time.perf_counter()
        logits = rt.forward(req["ids"], req["markers"], q)
        print(json.dumps(result_line(logits, 1e3 * (time.perf_counter() - t0))), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
