"""The registry wired into a Hugging Face decoder: a randomly initialised Qwen3
(Qwen3-0.6B layer shapes, 4 layers, built with ``from_config``; no checkpoint)
decodes through ``MultiDeltaLoRAModel`` with every projection on the W8A16
kernel (reference ``src/blackwell_inference/lora/delta_multi.py:20-89`` and
``serve/models.py:69-96``, which load Qwen3 checkpoints).

* Prefill logits of the wrapped fp16 model against the same model in fp32 with
  each projection's weight set to the dequantised int8 copy the layer uses
  (``q * scale``): the kernel path and torch's matmul agree within fp16
  activation rounding.
* With an adapter: logits follow the adapter's own int8 copy (and differ from
  the base), switching a -> b -> a gives bit-identical logits (no drift), and
  greedy decoding is deterministic.
"""
import copy

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
transformers = pytest.importorskip("transformers")

TARGETS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def _model(dev):
    from transformers import AutoModelForCausalLM, Qwen3Config

    cfg = Qwen3Config(hidden_size=1024, intermediate_size=3072, num_hidden_layers=4, num_attention_heads=16,
                      num_key_value_heads=8, head_dim=128, vocab_size=151936, tie_word_embeddings=True,
                      max_position_embeddings=4096)
    torch.manual_seed(0)
    return AutoModelForCausalLM.from_config(cfg).to(dev, torch.float16).eval()


def _adapter(model, r, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    out = {}
    for name, mod in model.named_modules():
        if isinstance(mod, torch.nn.Linear) and any(name.endswith(t) for t in TARGETS):
            n, k = mod.weight.shape
            A = (torch.randn(r, k, generator=g, device=dev) / k ** 0.5).half()
            B = (torch.randn(n, r, generator=g, device=dev) * 0.05).half()
            out[name] = (A, B, 2.0)
    return out


def _fp32_twin(fp16_model, mdl, adapter):
    """fp32 copy of the model whose projections hold the dequantised int8 copy of `adapter`."""
    twin = copy.deepcopy(fp16_model).float()
    for name, layer in mdl._lora_layers.items():
        q, s = layer.copies[adapter]
        parent_name, _, attr = name.rpartition(".")
        lin = torch.nn.Linear(layer.in_features, layer.out_features, bias=False, device=q.device)
        lin.weight.data = q.float() * s.float()[:, None]
        setattr(twin.get_submodule(parent_name), attr, lin)
    return twin


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm())


def test_qwen3_decode_through_registry(cuda_dev):
    from blackwell_inference.lora import MultiDeltaLoRAModel
    from blackwell_inference.lora.delta_multi import W8A16Linear

    model = _model(cuda_dev)
    plain = copy.deepcopy(model)
    mdl = MultiDeltaLoRAModel(model, device=str(cuda_dev), quantize=True)
    assert len(mdl.layer_names) == 4 * 7
    assert all(isinstance(mdl.base.get_submodule(n), W8A16Linear) for n in mdl.layer_names)

    ids = torch.randint(0, 151936, (2, 24), generator=torch.Generator().manual_seed(1)).to(cuda_dev)
    with torch.no_grad():
        base_logits = mdl(input_ids=ids, adapter=None).logits
        twin = _fp32_twin(plain, mdl, None)
        want = twin(input_ids=ids).logits
    assert _rel(base_logits, want) <= 2e-2, _rel(base_logits, want)

    assert mdl.load_adapter("a", _adapter(plain, 16, 11, cuda_dev)) == 28
    assert mdl.load_adapter("b", _adapter(plain, 64, 12, cuda_dev)) == 28
    with torch.no_grad():
        la = mdl(input_ids=ids, adapter="a").logits
        want_a = _fp32_twin(plain, mdl, "a")(input_ids=ids).logits
        lb = mdl(input_ids=ids, adapter="b").logits
        la2 = mdl(input_ids=ids, adapter="a").logits
    assert _rel(la, want_a) <= 2e-2, _rel(la, want_a)
    assert _rel(la, base_logits) > 0.1  # the adapter is applied
    assert _rel(lb, la) > 0.1
    assert torch.equal(la, la2), "switching adapters changed the logits"

    out1 = mdl.generate_ids(ids[:1, :8], adapter="a", max_new_tokens=8)
    out2 = mdl.generate_ids(ids[:1, :8], adapter="a", max_new_tokens=8)
    assert out1.shape[0] == 1 and 1 <= out1.shape[1] <= 8 and torch.equal(out1, out2)
    from blackwell_ops import _lib

    assert _lib.device_status() == 0
