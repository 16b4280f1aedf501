"""Additive memory adapter around Hugging Face decoder attentions.

Same interface and behaviour as the reference's compatibility adapter
(``src/hf_wrappers/pra_wrapper.py:12-112``): it keeps the pretrained attention and
adds ``alpha * cross_attention(hidden, retrieved blocks)``.  Retrieval is a toy
embedding index (mean input embedding per text block, cosine top-k with a
threshold); it has no URI / chunk provenance and no layer-specific K/V, so claims
about PRA itself belong to the native patch (``pdattention_b200.hf.convert``).
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F


class SimpleHFMemoryIndex:
    """Embeds every memory text once with the model's input embedding table."""

    def __init__(self, memory_texts, tokenizer, model, device, max_tokens: int = 256):
        self.memory_texts = list(memory_texts)
        self.tokenizer = tokenizer
        self.model = model
        self.device = device
        self.max_tokens = max_tokens
        self.memory_hidden: list[torch.Tensor] = []
        self.content_routing_vectors: torch.Tensor | None = None
        self.build()

    @torch.no_grad()
    def build(self) -> None:
        table = self.model.get_input_embeddings()
        blocks, keys = [], []
        for text in self.memory_texts:
            ids = self.tokenizer(text, return_tensors="pt", truncation=True,
                                 max_length=self.max_tokens).input_ids.to(self.device)
            hidden = table(ids)[0].detach()
            blocks.append(hidden)
            keys.append(hidden.mean(dim=0))
        self.memory_hidden = blocks
        self.content_routing_vectors = torch.stack(keys) if keys else None

    def search(self, query: torch.Tensor, top_k: int = 2, threshold: float = 0.2):
        """``query`` ``[1, D]`` -> the passing blocks concatenated ``[1, M, D]`` (or None)."""
        if self.content_routing_vectors is None:
            return None
        q = F.normalize(query[0].detach(), dim=-1)
        keys = F.normalize(self.content_routing_vectors.to(q.device), dim=-1)
        scores = keys @ q
        values, order = torch.topk(scores, k=min(top_k, len(self.memory_hidden)))
        picked = [self.memory_hidden[int(i)].to(q.device) for v, i in zip(values, order) if float(v) >= threshold]
        return torch.cat(picked).unsqueeze(0) if picked else None


class PRAAttentionAdapter(nn.Module):
    """``original(hidden) + alpha * o(softmax(q k^T / sqrt(D)) v)`` over retrieved blocks."""

    def __init__(self, original_attn, hidden_size, memory_index, alpha: float = 0.05, top_k: int = 2,
                 threshold: float = 0.2):
        super().__init__()
        self.original_attn = original_attn
        self.memory_index = memory_index
        self.alpha = alpha
        self.top_k = top_k
        self.threshold = threshold
        self.mem_q = nn.Linear(hidden_size, hidden_size, bias=False)
        self.mem_k = nn.Linear(hidden_size, hidden_size, bias=False)
        self.mem_v = nn.Linear(hidden_size, hidden_size, bias=False)
        self.mem_o = nn.Linear(hidden_size, hidden_size, bias=False)

    def forward(self, hidden_states, *args, **kwargs):
        result = self.original_attn(hidden_states, *args, **kwargs)
        base, rest = (result[0], result[1:]) if isinstance(result, tuple) else (result, ())
        # the final position routes; every position then attends to the retrieved blocks
        blocks = self.memory_index.search(hidden_states[:, -1, :], self.top_k, self.threshold)
        if blocks is None:
            return result
        blocks = blocks.to(hidden_states.device, hidden_states.dtype)
        q, k, v = self.mem_q(hidden_states), self.mem_k(blocks), self.mem_v(blocks)
        weights = torch.softmax(q @ k.transpose(-1, -2) / (q.shape[-1] ** 0.5), dim=-1)
        mixed = base + self.alpha * self.mem_o(weights @ v)
        return (mixed, *rest) if isinstance(result, tuple) else mixed


def patch_decoder_layers(model, memory_index, layer_ids, alpha: float = 0.05):
    """Wrap ``model.model.layers[i].self_attn`` for each ``i`` in ``layer_ids``."""
    hidden = model.config.hidden_size
    for layer_id in layer_ids:
        layer = model.model.layers[layer_id]
        layer.self_attn = PRAAttentionAdapter(layer.self_attn, hidden, memory_index, alpha=alpha)
    return model
