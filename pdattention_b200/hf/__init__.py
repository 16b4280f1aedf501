"""Hugging Face integration.

* ``adapter``: the compatibility adapter of the reference's HF path
  (``src/hf_wrappers/pra_wrapper.py``): an embedding-level memory index and an
  additive cross-attention branch wrapped around selected decoder attentions.
* ``convert``: the native-K/V PRA patch for Llama / Mistral / Qwen2 checkpoints:
  an HF model's weights become a ``PRALlamaReference`` (fp32 oracle) or the
  device engine's ``LlamaWeights``.
"""

from .adapter import PRAAttentionAdapter, SimpleHFMemoryIndex, patch_decoder_layers
from .convert import engine_from_hf, reference_from_hf

__all__ = ["PRAAttentionAdapter", "SimpleHFMemoryIndex", "patch_decoder_layers", "engine_from_hf",
           "reference_from_hf"]
