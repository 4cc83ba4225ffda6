"""Greedy-decode throughput of a Hugging Face decoder on the W8A16 registry.

The reference reports tokens/s of Qwen3 checkpoints served with and without
its LoRA path (README tok/s table).  No checkpoint is available here, so the
model is ``from_config`` with random weights at the named architecture's
shapes; the timings do not depend on weight values.  Both arms run
``transformers``' own eager ``generate`` at batch 1 (greedy, KV cache), so at
this size they mostly measure per-token launch overhead:

* ``fp16``: the model as loaded (torch linear layers);
* ``w8a16``: ``MultiDeltaLoRAModel(quantize=True)`` with one adapter loaded and
  active (every projection on the tcgen05 W8A16 GEMM).

``python -m blackwell_inference.decode_bench [--layers 28] [--tokens 64]``
prints one JSON line.
"""
from __future__ import annotations

import argparse
import copy
import json

import torch

QWEN3_0_6B = dict(hidden_size=1024, intermediate_size=3072, num_attention_heads=16, num_key_value_heads=8,
                  head_dim=128, vocab_size=151936, tie_word_embeddings=True, max_position_embeddings=4096)


def _tok_s(gen, ids, tokens: int, reps: int) -> float:
    gen(ids, 4)  # warm-up
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 0
    a.record()
    for _ in range(reps):
        n += gen(ids, tokens).shape[1]
    b.record()
    torch.cuda.synchronize()
    return n / (a.elapsed_time(b) / 1e3)


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=28)
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--rank", type=int, default=16)
    args = ap.parse_args(argv)
    from transformers import AutoModelForCausalLM, Qwen3Config

    from blackwell_inference.lora import MultiDeltaLoRAModel

    dev = torch.device("cuda", torch.cuda.current_device())
    torch.manual_seed(0)
    cfg = Qwen3Config(num_hidden_layers=args.layers, **QWEN3_0_6B)
    model = AutoModelForCausalLM.from_config(cfg).to(dev, torch.float16).eval()
    ids = torch.randint(0, cfg.vocab_size, (1, 16), generator=torch.Generator().manual_seed(3)).to(dev)

    def hf_gen(m):
        def gen(x, t):
            with torch.no_grad():
                out = m.generate(input_ids=x, attention_mask=torch.ones_like(x), max_new_tokens=t,
                                 min_new_tokens=t, do_sample=False)
            return out[:, x.shape[1]:]
        return gen

    fp16 = _tok_s(hf_gen(model), ids, args.tokens, args.reps)
    wrapped = MultiDeltaLoRAModel(copy.deepcopy(model), device=str(dev), quantize=True)
    del model
    wrapped.load_adapter("a", _adapter(wrapped, args.rank, dev))
    wrapped.set_adapter("a")
    w8 = _tok_s(hf_gen(wrapped.base), ids, args.tokens, args.reps)
    line = {"metric": "greedy decode tokens/s (batch 1, eager HF generate)", "unit": "tok/s",
            "model": f"Qwen3-0.6B shapes, {args.layers} layers, random init (from_config)",
            "tokens": args.tokens, "reps": args.reps, "fp16": round(fp16, 2), "w8a16_adapter": round(w8, 2),
            "adapter_rank": args.rank, "projections_on_w8a16": len(wrapped.layer_names)}
    print(json.dumps(line), flush=True)
    return line


def _adapter(mdl, r: int, dev) -> dict:
    """A random rank-r adapter for every projection the registry wrapped."""
    g = torch.Generator(device=dev).manual_seed(7)
    out = {}
    for name, layer in mdl._lora_layers.items():
        n, k = layer.out_features, layer.in_features
        out[name] = ((torch.randn(r, k, generator=g, device=dev) / k ** 0.5).half(),
                     (torch.randn(n, r, generator=g, device=dev) * 0.01).half(), 2.0)
    return out


if __name__ == "__main__":
    main()
