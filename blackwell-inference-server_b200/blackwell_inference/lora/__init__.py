from .delta_multi import MultiDeltaLoRAModel, W8A16Linear, read_peft_adapter

__all__ = ["MultiDeltaLoRAModel", "W8A16Linear", "read_peft_adapter"]
