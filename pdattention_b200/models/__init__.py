"""Model families: TinyGPT-PRA (standalone) and the PRA-patched Llama family."""

from .attention import PRAttention
from .tiny import (
    PRASATransformerBlock,
    PRATransformerBlock,
    TinyPRALanguageModel,
    TinyPRAModel,
    TransformerBlock,
    VanillaTransformerBlock,
    causal_attention_mask,
    convert_sa_checkpoint_to_pra,
    convert_sa_model_to_pra,
)

__all__ = [name for name in dir() if not name.startswith("_")]
