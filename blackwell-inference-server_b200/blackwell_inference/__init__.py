"""blackwell_inference (B200 edition): the LoRA registry that serves adapters on
the W8A16 / LoRA-delta operators of ``blackwell_ops``."""
