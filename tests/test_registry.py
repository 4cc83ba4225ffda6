"""LoRA registry (blackwell_inference.lora.delta_multi) on the B200 operators.

CPU: PEFT adapter-directory parsing.  GPU: per-adapter int8 copies are exactly
quantize(merge(W, A, B)), forward runs the W8A16 kernel, and switching
adapters never drifts (the reference's `weight -= old; weight += new` does).
"""
import json

import numpy as np
import pytest
import torch

TARGETS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
SHAPES = {"q_proj": (256, 512), "k_proj": (256, 128), "v_proj": (256, 128), "o_proj": (512, 256),
          "gate_proj": (256, 768), "up_proj": (256, 768), "down_proj": (768, 256)}


class TinyLayer(torch.nn.Module):
    def __init__(self):
        super().__init__()
        for name, (k, n) in SHAPES.items():
            setattr(self, name, torch.nn.Linear(k, n, bias=False))


class TinyModel(torch.nn.Module):
    def __init__(self, layers=2):
        super().__init__()
        self.layers = torch.nn.ModuleList([TinyLayer() for _ in range(layers)])
        self.head = torch.nn.Linear(256, 64, bias=True)  # not a target

    def forward(self, x):
        outs = {}
        for i, layer in enumerate(self.layers):
            for name in TARGETS:
                k, _ = SHAPES[name]
                outs[f"layers.{i}.{name}"] = getattr(layer, name)(x[..., :k] if x.shape[-1] >= k else
                                                                     torch.nn.functional.pad(x, (0, k - x.shape[-1])))
        return outs


def make_model(seed=0):
    torch.manual_seed(seed)
    m = TinyModel()
    with torch.no_grad():
        for p in m.parameters():
            p.mul_(0.05)
    return m.half()


def make_adapter(n_layers, r, seed, alpha=None):
    g = torch.Generator().manual_seed(seed)
    alpha = alpha if alpha is not None else 2 * r
    out = {}
    for i in range(n_layers):
        for name in TARGETS:
            k, n = SHAPES[name]
            A = (torch.randn(r, k, generator=g) / k ** 0.5).half()
            B = (torch.randn(n, r, generator=g) * 0.01).half()
            out[f"layers.{i}.{name}"] = (A, B, alpha / r)
    return out


def test_read_peft_adapter_directory(tmp_path):
    from safetensors.torch import save_file

    from blackwell_inference.lora import read_peft_adapter

    r, alpha = 8, 32
    tensors = {
        "base_model.model.model.layers.0.self_attn.q_proj.lora_A.weight": torch.randn(r, 64).half(),
        "base_model.model.model.layers.0.self_attn.q_proj.lora_B.weight": torch.randn(128, r).half(),
        "base_model.model.model.layers.3.mlp.down_proj.lora_A.weight": torch.randn(r, 256).half(),
        "base_model.model.model.layers.3.mlp.down_proj.lora_B.weight": torch.randn(64, r).half(),
    }
    save_file(tensors, str(tmp_path / "adapter_model.safetensors"))
    (tmp_path / "adapter_config.json").write_text(json.dumps({"r": r, "lora_alpha": alpha,
                                                              "target_modules": ["q_proj", "down_proj"]}))
    cfg, entries = read_peft_adapter(tmp_path)
    assert cfg["r"] == r
    assert set(entries) == {"model.layers.0.self_attn.q_proj", "model.layers.3.mlp.down_proj"}
    A, B, s = entries["model.layers.0.self_attn.q_proj"]
    assert A.shape == (r, 64) and B.shape == (128, r) and s == alpha / r
    (tmp_path / "adapter_config.json").write_text(json.dumps({"r": r, "lora_alpha": alpha, "use_rslora": True}))
    _, entries = read_peft_adapter(tmp_path)
    assert abs(entries["model.layers.3.mlp.down_proj"][2] - alpha / r ** 0.5) < 1e-12


@pytest.mark.gpu
def test_registry_int8_copies_and_switching(cuda_dev):
    from blackwell_inference.lora import MultiDeltaLoRAModel
    from blackwell_ops.cuda import lora_merge
    from blackwell_ops.kernels import int8_gemm, quantize_weight_int8

    model = make_model()
    base_w = {n: m.weight.detach().clone() for n, m in model.named_modules() if isinstance(m, torch.nn.Linear)}
    reg = MultiDeltaLoRAModel(model, device="cuda")
    assert len(reg.layer_names) == 14
    ad1, ad2 = make_adapter(2, 16, 1), make_adapter(2, 128, 2)
    assert reg.load_adapter("a", ad1) == 14
    assert reg.load_adapter("b", ad2) == 14
    x = torch.randn(3, 5, 256, device=cuda_dev).half()
    outs = {}
    for name in (None, "a", "b", "a", None, "b"):
        outs.setdefault(name, []).append(reg(x, adapter=name))
    for name, runs in outs.items():  # no drift across switches
        for o in runs[1:]:
            for key in o:
                assert torch.equal(o[key], runs[0][key]), (name, key)
    # every adapter copy is exactly quantize(merge(W, A, B, s)); forward is the W8A16 kernel on it
    layer_name = "layers.1.gate_proj"
    layer = reg.base.get_submodule(layer_name)
    W = base_w[layer_name].to(cuda_dev)
    A, B, s = ad1[layer_name]
    q, sc = quantize_weight_int8(lora_merge(W, A.to(cuda_dev), B.to(cuda_dev), s))
    assert torch.equal(layer.copies["a"][0], q) and torch.equal(layer.copies["a"][1], sc)
    y = int8_gemm(x.reshape(-1, 256), q, sc).reshape(3, 5, -1)
    assert torch.equal(outs["a"][0][layer_name], y)
    # and it is close to the unquantised merged linear
    ref = x.double() @ (W.double() + s * B.double().to(cuda_dev) @ A.double().to(cuda_dev)).t()
    assert float((y.double() - ref).abs().max()) < 0.05


@pytest.mark.gpu
def test_registry_fp16_mode_is_drift_free(cuda_dev):
    from blackwell_inference.lora import MultiDeltaLoRAModel
    from blackwell_ops.cuda import lora_merge

    model = make_model(3)
    reg = MultiDeltaLoRAModel(model, device="cuda", quantize=False, targets=("q_proj", "v_proj"))
    ad = make_adapter(2, 16, 5)
    ad2 = make_adapter(2, 16, 6)
    reg.load_adapter("x", {k: v for k, v in ad.items() if "q_proj" in k or "v_proj" in k})
    reg.load_adapter("y", {k: v for k, v in ad2.items() if "q_proj" in k or "v_proj" in k})
    name = "layers.0.q_proj"
    mod = reg.base.get_submodule(name)
    base = mod.weight.detach().clone()
    A, B, s = ad[name]
    want = lora_merge(base, A.to(cuda_dev), B.to(cuda_dev), s)
    for _ in range(20):
        reg.set_adapter("x")
        reg.set_adapter("y")
    reg.set_adapter("x")
    assert torch.equal(mod.weight, want)
    reg.set_adapter(None)
    assert torch.equal(mod.weight, base)
    # the reference's switching (weight -= old; weight += new, delta_multi.py:71,75) drifts
    w = base.clone()
    d1 = ((B.float() @ A.float()) * s).half().to(cuda_dev)
    A2, B2, s2 = ad2[name]
    d2 = ((B2.float() @ A2.float()) * s2).half().to(cuda_dev)
    w += d1
    for _ in range(20):
        w -= d1
        w += d2
        w -= d2
        w += d1
    assert not torch.equal(w, base + d1)
