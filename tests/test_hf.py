"""Hugging Face integration on CPU: the compatibility adapter and the native patch."""

import pytest
import torch

transformers = pytest.importorskip("transformers")


class _Tok:
    """Word-id tokenizer with the HF call signature the adapter uses."""

    def __call__(self, text, return_tensors="pt", truncation=True, max_length=256):
        ids = [hash(w) % 97 + 3 for w in text.split()][:max_length]
        return type("Enc", (), {"input_ids": torch.tensor([ids])})()


def _tiny(model_type):
    common = dict(vocab_size=128, hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                  num_key_value_heads=2, max_position_embeddings=256)
    cfg = transformers.Qwen2Config(**common) if model_type == "qwen2" else transformers.LlamaConfig(**common)
    cfg._attn_implementation = "eager"
    cls = transformers.Qwen2ForCausalLM if model_type == "qwen2" else transformers.LlamaForCausalLM
    torch.manual_seed(0)
    return cls(cfg).eval()


def test_adapter_patches_layers_and_keeps_outputs_shape():
    from pdattention_b200.hf import SimpleHFMemoryIndex, patch_decoder_layers

    model = _tiny("qwen2")
    ids = torch.randint(0, 128, (1, 7))
    with torch.no_grad():
        before = model(ids).logits
    index = SimpleHFMemoryIndex(["alpha beta gamma", "delta epsilon"], _Tok(), model, "cpu")
    assert index.content_routing_vectors.shape == (2, 64)
    patch_decoder_layers(model, index, layer_ids=[-1], alpha=0.5)
    with torch.no_grad():
        after = model(ids).logits
    assert after.shape == before.shape
    blocks = index.search(model.get_input_embeddings()(ids)[:, -1, :], top_k=2, threshold=-1.0)
    assert blocks is not None and blocks.shape[0] == 1
    # threshold above every cosine: nothing retrieved, the wrapped attention is unchanged
    model.model.layers[-1].self_attn.threshold = 2.0
    with torch.no_grad():
        same = model(ids).logits
    assert torch.allclose(same, before, atol=1e-6)


@pytest.mark.parametrize("model_type", ["llama", "qwen2"])
def test_native_patch_loads_hf_weights(model_type):
    from pdattention_b200.hf import reference_from_hf

    hf = _tiny(model_type)
    ours = reference_from_hf(hf, chunk_tokens=8, top_k_chunks=2)
    ids = torch.randint(0, 128, (2, 9))
    with torch.no_grad():
        ref = hf(ids).logits
    assert torch.allclose(ours(ids), ref, atol=1e-4)
