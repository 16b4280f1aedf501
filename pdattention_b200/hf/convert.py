"""Native-K/V PRA patch for Hugging Face Llama / Mistral / Qwen2 models.

The PRA Llama-family models keep the Hugging Face parameter layout, so an HF model
(or its state dict) becomes a ``PRALlamaReference`` by a plain state-dict load, and
the device engine's bf16 ``LlamaWeights`` (optionally one tensor-parallel shard)
from that.  RoPE, GQA and the per-layer K/V cache are the engine's own.
"""

from __future__ import annotations

from ..models.llama import PRALlamaConfig, PRALlamaReference


def config_from_hf(hf_config, **pra) -> PRALlamaConfig:
    family = {"llama": "llama", "mistral": "mistral", "qwen2": "qwen2"}.get(hf_config.model_type)
    if family is None:
        raise ValueError(f"unsupported model type {hf_config.model_type!r} (llama, mistral or qwen2)")
    heads = hf_config.num_attention_heads
    head_dim = getattr(hf_config, "head_dim", None) or hf_config.hidden_size // heads
    return PRALlamaConfig(
        family=family, vocab_size=hf_config.vocab_size, hidden_size=hf_config.hidden_size,
        intermediate_size=hf_config.intermediate_size, num_hidden_layers=hf_config.num_hidden_layers,
        num_attention_heads=heads, num_key_value_heads=hf_config.num_key_value_heads, head_dim=head_dim,
        rope_theta=float(getattr(hf_config, "rope_theta", None) or
                         (getattr(hf_config, "rope_parameters", None) or {}).get("rope_theta", 10000.0)),
        rms_norm_eps=hf_config.rms_norm_eps,
        attention_bias=bool(getattr(hf_config, "attention_bias", family == "qwen2")),
        tie_word_embeddings=bool(getattr(hf_config, "tie_word_embeddings", False)),
        max_position_embeddings=hf_config.max_position_embeddings, **pra)


def reference_from_hf(hf_model, **pra) -> PRALlamaReference:
    """fp32 PRA model carrying the HF model's weights."""
    cfg = config_from_hf(hf_model.config, **pra)
    model = PRALlamaReference(cfg)
    state = {k: v.float() for k, v in hf_model.state_dict().items() if "rotary_emb" not in k}
    if cfg.tie_word_embeddings:
        state.pop("lm_head.weight", None)
    model.load_state_dict(state, strict=True)
    return model.eval()


def engine_from_hf(hf_model, device, tp=None, **pra):
    """A device engine (this rank's shard when ``tp`` is given) for an HF model."""
    from ..inference.llama_engine import LlamaWeights, PRALlamaEngine

    reference = reference_from_hf(hf_model, **pra)
    rank, size = (tp.rank, tp.world) if tp is not None else (0, 1)
    return PRALlamaEngine(LlamaWeights.from_reference(reference, device, rank, size), device, tp=tp)
