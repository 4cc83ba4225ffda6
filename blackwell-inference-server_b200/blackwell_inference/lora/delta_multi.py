"""Multi-LoRA serving on the B200 W8A16 / LoRA-delta operators.

Drop-in for the reference's ``MultiDeltaLoRAModel``
(``src/blackwell_inference/lora/delta_multi.py:20-89``): one base model, any
number of adapters, ``load_adapter(name, path)`` and
``generate(prompt, adapter=...)``.  The reference keeps one fp16 delta per
adapter and layer, computed with ``(B @ A) * scaling`` in plain torch (``:59``),
and switches adapters by ``weight -= old; weight += new`` (``:65-76``), which
re-rounds the fp16 weight on every switch (the weights drift).

Here every adapted projection becomes a :class:`W8A16Linear` whose forward is
the tcgen05 ``int8_gemm``:

* ``quantize=True`` (default): each adapter is merged into its OWN int8 copy
  of the projection with the fused ``lora_merge_requant`` (delta, merge and
  per-channel requantisation in one kernel, the merged fp16 weight never
  written).  Switching adapters swaps which (int8, scale) pair the layer
  reads: no arithmetic, no drift.
* ``quantize=False``: fp16 weights as in the reference, but the live weight is
  recomputed from the untouched base with the fused ``lora_merge`` on each
  switch, so switching never drifts.

The projections adapted by default are all seven of a decoder layer (the
reference adapts q/k/v/o only, ``:35-40``); pass ``targets`` to narrow them.
Adapters can be loaded from a PEFT adapter directory (``adapter_config.json``
+ ``adapter_model.safetensors``, read without the ``peft`` package) or from a
``{layer_name: (A, B, scaling)}`` mapping.
"""
from __future__ import annotations

import json
import math
from pathlib import Path
from typing import Iterable, Mapping

import torch

DEFAULT_TARGETS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


class W8A16Linear(torch.nn.Module):
    """``nn.Linear`` replacement computing ``x @ (q * scale).T + bias`` with the W8A16 kernel.

    Holds the fp16 base weight (to merge new adapters from), its int8
    quantisation, and one (int8, scale) pair per loaded adapter.
    """

    def __init__(self, linear: torch.nn.Linear, keep_base: bool = True):
        super().__init__()
        from blackwell_ops.kernels import quantize_weight_int8

        w = linear.weight.detach()
        if w.dtype != torch.float16:
            w = w.to(torch.float16)
        self.in_features = linear.in_features
        self.out_features = linear.out_features
        self.base_weight = w.contiguous() if keep_base else None
        self.bias = linear.bias
        q, s = quantize_weight_int8(w)
        self.copies: dict[str | None, tuple[torch.Tensor, torch.Tensor]] = {None: (q, s)}
        self.active: str | None = None

    def add_adapter(self, name: str, A: torch.Tensor, B: torch.Tensor, scaling: float) -> None:
        from blackwell_ops.cuda import lora_merge_requant

        if self.base_weight is None:
            raise RuntimeError("this layer was built without its fp16 base weight; cannot merge adapters")
        dev = self.base_weight.device
        q, s = lora_merge_requant(self.base_weight, A.to(dev, torch.float16), B.to(dev, torch.float16), scaling)
        self.copies[name] = (q, s)

    def remove_adapter(self, name: str) -> None:
        if name is not None:
            self.copies.pop(name, None)
            if self.active == name:
                self.active = None

    def set_adapter(self, name: str | None) -> None:
        self.active = name if name in self.copies else None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        from blackwell_ops.kernels import int8_gemm

        q, s = self.copies[self.active]
        x2 = x.reshape(-1, self.in_features)
        if x2.dtype not in (torch.float16, torch.bfloat16):
            x2 = x2.to(torch.float16)
        y = int8_gemm(x2, q, s).reshape(*x.shape[:-1], self.out_features)
        if self.bias is not None:
            y = y + self.bias.to(y.dtype)
        return y.to(x.dtype) if x.dtype != y.dtype else y


def read_peft_adapter(path: str | Path) -> tuple[dict, dict[str, tuple[torch.Tensor, torch.Tensor, float]]]:
    """Read a PEFT LoRA adapter directory without the ``peft`` package.

    Returns ``(config, {module_name: (A [r, in], B [out, r], scaling)})`` where
    module names are relative to the base model (the ``base_model.model.``
    prefix PEFT adds is stripped) and ``scaling = lora_alpha / r`` (``/ sqrt(r)``
    with rsLoRA), as PEFT computes it.
    """
    from safetensors.torch import load_file

    path = Path(path)
    cfg = json.loads((path / "adapter_config.json").read_text())
    tensors = load_file(str(path / "adapter_model.safetensors"))
    r = int(cfg["r"])
    alpha = float(cfg.get("lora_alpha", r))
    scaling = alpha / math.sqrt(r) if cfg.get("use_rslora") else alpha / r
    pairs: dict[str, dict[str, torch.Tensor]] = {}
    for key, t in tensors.items():
        for part in ("lora_A", "lora_B"):
            tag = f".{part}."
            if tag in key:
                mod = key.split(tag)[0]
                for prefix in ("base_model.model.",):
                    if mod.startswith(prefix):
                        mod = mod[len(prefix):]
                pairs.setdefault(mod, {})[part] = t
    out = {m: (p["lora_A"], p["lora_B"], scaling) for m, p in pairs.items() if "lora_A" in p and "lora_B" in p}
    return cfg, out


class MultiDeltaLoRAModel:
    """One base model + per-adapter merged weights; adapter switching without drift.

    ``base`` is a model path (loaded with transformers in fp16, as the
    reference does) or an existing ``torch.nn.Module``.
    """

    def __init__(self, base: str | torch.nn.Module, device: str = "cuda", tokenizer=None,
                 targets: Iterable[str] = DEFAULT_TARGETS, quantize: bool = True, exact: bool = False):
        self.device = device
        self.quantize = quantize
        # exact=True: adapters merged with the reference's own accumulation order (CUDA cores), so
        # every int8 copy equals quantize_weight_int8(add_delta_(W, lora_delta(A, B, s))) bit for bit
        self.exact = exact
        self.targets = tuple(targets)
        if isinstance(base, (str, Path)):
            from transformers import AutoModelForCausalLM, AutoTokenizer

            self.base_model_path = str(base)
            self.tokenizer = AutoTokenizer.from_pretrained(self.base_model_path)
            self.base = AutoModelForCausalLM.from_pretrained(self.base_model_path, torch_dtype=torch.float16,
                                                             device_map=device)
        else:
            self.base_model_path = None
            self.tokenizer = tokenizer
            self.base = base.to(device)
        self._lora_layers: dict[str, torch.nn.Module] = {}
        self._fp16_base: dict[str, torch.Tensor] = {}
        self._adapters: dict[str, dict[str, tuple[torch.Tensor, torch.Tensor, float]]] = {}
        self._current_adapter: str | None = None
        self._collect_lora_layers()

    # ---- layer discovery (reference :35-40) ----
    def _collect_lora_layers(self) -> None:
        found = [(n, m) for n, m in self.base.named_modules()
                 if isinstance(m, torch.nn.Linear) and any(t in n for t in self.targets)]
        for name, module in found:
            if self.quantize:
                parent_name, _, attr = name.rpartition(".")
                parent = self.base.get_submodule(parent_name) if parent_name else self.base
                layer = W8A16Linear(module)
                setattr(parent, attr, layer)
                self._lora_layers[name] = layer
            else:
                if module.weight.dtype != torch.float16:
                    module.to(torch.float16)
                self._fp16_base[name] = module.weight.detach().clone()
                self._lora_layers[name] = module

    @property
    def layer_names(self) -> list[str]:
        return list(self._lora_layers)

    # ---- adapters (reference :42-63) ----
    def load_adapter(self, name: str, adapter: str | Path | Mapping[str, tuple]) -> int:
        """Load an adapter from a PEFT directory or a {layer: (A, B, scaling)} mapping.

        Returns the number of layers the adapter touches.
        """
        if isinstance(adapter, (str, Path)):
            _, entries = read_peft_adapter(adapter)
        else:
            entries = dict(adapter)
        used: dict[str, tuple[torch.Tensor, torch.Tensor, float]] = {}
        for layer_name in self._lora_layers:
            if layer_name not in entries:
                continue
            A, B, scaling = entries[layer_name]
            A = A.to(self.device, torch.float16).contiguous()
            B = B.to(self.device, torch.float16).contiguous()
            used[layer_name] = (A, B, float(scaling))
        if self.quantize and used:
            # every projection of the adapter merged + requantised in batched launches
            from blackwell_ops.cuda import lora_merge_requant_batched

            names = list(used)
            layers = [self._lora_layers[n] for n in names]
            for layer in layers:
                if layer.base_weight is None:
                    raise RuntimeError("a layer was built without its fp16 base weight; cannot merge adapters")
            outs = lora_merge_requant_batched(
                ((layer.base_weight, used[n][0], used[n][1], used[n][2]) for n, layer in zip(names, layers)),
                exact=self.exact)
            # adapter loading is not on the serving path: synchronise and raise if a device wait of
            # the batched requantisation ran out (its codes would be incomplete)
            from blackwell_ops.device import check

            check(layers[0].base_weight.device, f"load_adapter({name!r})")
            for layer, (q, s) in zip(layers, outs):
                layer.copies[name] = (q, s)
        self._adapters[name] = used
        if self._current_adapter == name:  # reloaded while active: re-apply
            self._current_adapter = None
            self._apply_delta(name)
        return len(used)

    def unload_adapter(self, name: str) -> None:
        if self._current_adapter == name:
            self._apply_delta(None)
        self._adapters.pop(name, None)
        if self.quantize:
            for layer in self._lora_layers.values():
                layer.remove_adapter(name)

    # ---- switching (reference :65-76), drift-free ----
    def _apply_delta(self, adapter_name: str | None) -> None:
        if self._current_adapter == adapter_name:
            return
        if adapter_name is not None and adapter_name not in self._adapters:
            raise KeyError(f"adapter {adapter_name!r} is not loaded")
        if self.quantize:
            for layer in self._lora_layers.values():
                layer.set_adapter(adapter_name)
        else:
            from blackwell_ops.cuda import lora_merge

            entries = self._adapters.get(adapter_name, {}) if adapter_name is not None else {}
            for layer_name, module in self._lora_layers.items():
                base = self._fp16_base[layer_name]
                if layer_name in entries:
                    A, B, s = entries[layer_name]
                    lora_merge(base, A, B, s, out=module.weight.data, exact=self.exact)
                else:
                    module.weight.data.copy_(base)
        self._current_adapter = adapter_name

    set_adapter = _apply_delta

    @property
    def current_adapter(self) -> str | None:
        return self._current_adapter

    def __call__(self, *args, adapter: str | None = None, **kwargs):
        self._apply_delta(adapter)
        with torch.no_grad():
            return self.base(*args, **kwargs)

    def generate_ids(self, input_ids: torch.Tensor, adapter: str | None = None, max_new_tokens: int = 64,
                     **kwargs) -> torch.Tensor:
        """Greedy decode from token ids (no tokenizer needed): the new tokens, [batch, <= max_new_tokens]."""
        self._apply_delta(adapter)
        input_ids = input_ids.to(self.device)
        with torch.no_grad():
            out = self.base.generate(input_ids=input_ids, attention_mask=torch.ones_like(input_ids),
                                     max_new_tokens=max_new_tokens, do_sample=False, **kwargs)
        return out[:, input_ids.shape[1]:]

    # ---- generation (reference :78-89) ----
    def generate(self, prompt: str, adapter: str | None = None, max_new_tokens: int = 64) -> str:
        if self.tokenizer is None:
            raise RuntimeError("generate() needs a tokenizer (load the model from a path or pass tokenizer=)")
        self._apply_delta(adapter)
        inputs = self.tokenizer(prompt, return_tensors="pt").to(self.device)
        with torch.no_grad():
            out = self.base.generate(**inputs, max_new_tokens=max_new_tokens, do_sample=False)
        return self.tokenizer.decode(out[0, inputs["input_ids"].shape[1]:], skip_special_tokens=True)
