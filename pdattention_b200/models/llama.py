"""PRA-patched Llama-family decoders (Llama 3, Mistral, Qwen2): configuration and fp32 oracle.

The reference ships no Llama-family PRA model: its HF path is a cross-attention
adapter (``src/hf_wrappers/pra_wrapper.py:58-112``) and ``src/llama_patch/README.md:7-17``
lists the constraints a real patch must keep (RoPE, GQA, the past-key-value cache).
This module defines the native-K/V PRA patch for these families:

* Architecture: RMSNorm, rotary positions (``rotate_half`` convention), grouped-query
  attention, SwiGLU MLP, optional q/k/v biases (Qwen2), untied or tied LM head.
  Parameter names follow the Hugging Face layout (``model.layers.{i}.self_attn.q_proj``
  ...), so such checkpoints load unchanged.
* Memory: every reference chunk is encoded as its own sequence (positions
  ``0..len-1``); each PRA layer keeps the chunk's post-rotary K/V (what the attention
  reads) and one routing gist, the mean of the chunk's PRE-rotary keys flattened over
  the KV heads (``[Hkv * Dh]``).  Routing compares content, not positions.
* Routing: the layer's routing query is the pre-rotary query of the routing token
  (the last valid prompt token, or the token being decoded) averaged over the query
  heads of each KV group, i.e. a ``[Hkv * Dh]`` vector in key space; the score is
  the cosine with each chunk gist (eps 1e-12, like ``memory.py:539-563``), and the
  ``top_k_chunks`` best chunks of the row's namespace are selected (ties broken by
  the lower chunk index), then materialised in chunk order.
* Attention: one softmax over ``[selected memory keys (all visible) ; local causal
  keys]`` per query head, the native-K/V transport of ``memory_batching.py:216-307``
  extended to GQA.

``PRALlamaReference`` is the fp32 oracle the device engine is tested against.
"""

from __future__ import annotations

import math
from dataclasses import asdict, dataclass, field

import torch
import torch.nn as nn
import torch.nn.functional as F

_FAMILIES = ("llama", "mistral", "qwen2")


@dataclass
class PRALlamaConfig:
    family: str = "llama"
    vocab_size: int = 128256
    hidden_size: int = 4096
    intermediate_size: int = 14336
    num_hidden_layers: int = 32
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    head_dim: int = 128
    rope_theta: float = 500000.0
    rms_norm_eps: float = 1e-5
    attention_bias: bool = False
    tie_word_embeddings: bool = False
    max_position_embeddings: int = 131072
    # PRA memory
    chunk_tokens: int = 64
    top_k_chunks: int = 16
    direct_window: int = 4096
    pra_layers: tuple | None = None   # layer ids that read memory (None: every layer)
    memory_budget_tokens: int | None = None  # cap on materialised memory tokens per row and layer

    def __post_init__(self):
        if self.family not in _FAMILIES:
            raise ValueError(f"family must be one of {_FAMILIES}")
        if self.num_attention_heads % self.num_key_value_heads:
            raise ValueError("num_attention_heads must be a multiple of num_key_value_heads")
        if self.head_dim % 2:
            raise ValueError("head_dim must be even (rotary pairs)")
        if self.top_k_chunks < 0 or self.chunk_tokens <= 0:
            raise ValueError("top_k_chunks must be >= 0 and chunk_tokens > 0")
        if self.pra_layers is not None:
            self.pra_layers = tuple(int(i) for i in self.pra_layers)

    @property
    def q_dim(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_key_value_heads * self.head_dim

    @property
    def group(self) -> int:
        return self.num_attention_heads // self.num_key_value_heads

    def is_pra_layer(self, layer: int) -> bool:
        return self.pra_layers is None or layer in self.pra_layers

    @property
    def memory_tokens_per_row(self) -> int:
        n = self.top_k_chunks * self.chunk_tokens
        return n if self.memory_budget_tokens is None else min(n, self.memory_budget_tokens)

    def to_dict(self) -> dict:
        return asdict(self)

    def parameter_count(self) -> int:
        d, f, v = self.hidden_size, self.intermediate_size, self.vocab_size
        attn = d * (self.q_dim + 2 * self.kv_dim) + self.q_dim * d
        if self.attention_bias:
            attn += self.q_dim + 2 * self.kv_dim
        per_layer = attn + 3 * d * f + 2 * d
        head = 0 if self.tie_word_embeddings else v * d
        return self.num_hidden_layers * per_layer + v * d + d + head


def llama3_8b(**kw) -> PRALlamaConfig:
    """Llama-3-8B architecture (random weights in this framework's benchmarks)."""
    return PRALlamaConfig(**{**dict(family="llama"), **kw})


def mistral_7b(**kw) -> PRALlamaConfig:
    """Mistral-7B (v0.3) architecture."""
    base = dict(family="mistral", vocab_size=32768, rope_theta=1000000.0, max_position_embeddings=32768)
    return PRALlamaConfig(**{**base, **kw})


def qwen2_7b(**kw) -> PRALlamaConfig:
    """Qwen2-7B architecture (q/k/v biases, 28 heads over 4 KV heads)."""
    base = dict(family="qwen2", vocab_size=152064, hidden_size=3584, intermediate_size=18944, num_hidden_layers=28,
                num_attention_heads=28, num_key_value_heads=4, head_dim=128, rope_theta=1000000.0,
                rms_norm_eps=1e-6, attention_bias=True, max_position_embeddings=32768)
    return PRALlamaConfig(**{**base, **kw})


def tiny_llama(**kw) -> PRALlamaConfig:
    """A small configuration of the same architecture for tests."""
    base = dict(vocab_size=256, hidden_size=128, intermediate_size=256, num_hidden_layers=2, num_attention_heads=4,
                num_key_value_heads=2, head_dim=32, rope_theta=10000.0, max_position_embeddings=2048,
                chunk_tokens=16, top_k_chunks=3, direct_window=256)
    return PRALlamaConfig(**{**base, **kw})


PRESETS = {"llama3-8b": llama3_8b, "mistral-7b": mistral_7b, "qwen2-7b": qwen2_7b, "tiny": tiny_llama}


# ---------------------------------------------------------------------------
# Rotary positions
# ---------------------------------------------------------------------------

def rope_tables(cfg: PRALlamaConfig, positions: torch.Tensor, dtype=torch.float32):
    """cos/sin ``[..., Dh]`` for integer ``positions`` (HF ``rotate_half`` layout)."""
    half = cfg.head_dim // 2
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, half, dtype=torch.float64, device=positions.device) / half))
    ang = positions.to(torch.float64)[..., None] * inv
    ang = torch.cat([ang, ang], dim=-1)
    return ang.cos().to(dtype), ang.sin().to(dtype)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """``x`` ``[B, T, H, Dh]``, cos/sin ``[B, T, Dh]``."""
    half = x.shape[-1] // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return x * cos[:, :, None, :] + rot * sin[:, :, None, :]


# ---------------------------------------------------------------------------
# Memory (oracle form)
# ---------------------------------------------------------------------------

@dataclass
class LlamaChunkMemory:
    """Encoded chunks: per layer post-rotary K/V and pre-rotary mean-key gists.

    ``k[l]``/``v[l]``: ``[C, chunk_tokens, Hkv, Dh]`` (rows past ``length[c]`` unused);
    ``gist[l]``: ``[C, Hkv * Dh]``; ``namespace[b]``: the chunk ids row ``b`` may read.
    """

    k: list = field(default_factory=list)
    v: list = field(default_factory=list)
    gist: list = field(default_factory=list)
    length: torch.Tensor | None = None
    namespace: list | None = None


def select_chunks(cfg: PRALlamaConfig, query: torch.Tensor, gist: torch.Tensor, namespace: list[list[int]]):
    """Cosine routing: ``query`` ``[B, kv_dim]`` against ``gist`` ``[C, kv_dim]`` -> per row
    the selected chunk ids in materialisation (chunk) order."""
    qn = F.normalize(query.float(), dim=-1, eps=1e-12)
    gn = F.normalize(gist.float(), dim=-1, eps=1e-12)
    out = []
    for b, ids in enumerate(namespace):
        if not ids or cfg.top_k_chunks == 0:
            out.append([])
            continue
        ids_t = torch.tensor(ids, dtype=torch.long, device=gist.device)
        scores = gn[ids_t] @ qn[b]
        order = sorted(range(len(ids)), key=lambda i: (-float(scores[i]), ids[i]))
        picked = [ids[i] for i in order[: cfg.top_k_chunks]]
        budget = cfg.memory_budget_tokens
        if budget is not None:
            kept, used = [], 0
            for c in picked:  # greedy whole chunks in score order
                n = cfg.chunk_tokens
                if used + n <= budget:
                    kept.append(c)
                    used += n
            picked = kept
        out.append(sorted(picked))
    return out


# ---------------------------------------------------------------------------
# fp32 oracle
# ---------------------------------------------------------------------------

class _RMSNorm(nn.Module):
    def __init__(self, d: int, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(d))
        self.eps = eps

    def forward(self, x):
        x32 = x.float()
        return (x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + self.eps)) * self.weight


class _Attention(nn.Module):
    def __init__(self, cfg: PRALlamaConfig):
        super().__init__()
        d = cfg.hidden_size
        self.q_proj = nn.Linear(d, cfg.q_dim, bias=cfg.attention_bias)
        self.k_proj = nn.Linear(d, cfg.kv_dim, bias=cfg.attention_bias)
        self.v_proj = nn.Linear(d, cfg.kv_dim, bias=cfg.attention_bias)
        self.o_proj = nn.Linear(cfg.q_dim, d, bias=False)


class _Mlp(nn.Module):
    def __init__(self, cfg: PRALlamaConfig):
        super().__init__()
        d, f = cfg.hidden_size, cfg.intermediate_size
        self.gate_proj = nn.Linear(d, f, bias=False)
        self.up_proj = nn.Linear(d, f, bias=False)
        self.down_proj = nn.Linear(f, d, bias=False)


class _Layer(nn.Module):
    def __init__(self, cfg: PRALlamaConfig):
        super().__init__()
        self.self_attn = _Attention(cfg)
        self.mlp = _Mlp(cfg)
        self.input_layernorm = _RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.post_attention_layernorm = _RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)


class _Body(nn.Module):
    def __init__(self, cfg: PRALlamaConfig):
        super().__init__()
        self.embed_tokens = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        self.layers = nn.ModuleList([_Layer(cfg) for _ in range(cfg.num_hidden_layers)])
        self.norm = _RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)


class PRALlamaReference(nn.Module):
    """fp32 PRA-Llama forward (prefill / full sequence) with optional chunk memory."""

    def __init__(self, cfg: PRALlamaConfig):
        super().__init__()
        self.cfg = cfg
        self.model = _Body(cfg)
        self.lm_head = None if cfg.tie_word_embeddings else nn.Linear(cfg.hidden_size, cfg.vocab_size, bias=False)
        self.reset_parameters()

    @torch.no_grad()
    def reset_parameters(self, std: float = 0.02, seed: int | None = None) -> None:
        gen = torch.Generator().manual_seed(seed) if seed is not None else None
        for name, p in self.named_parameters():
            if name.endswith("layernorm.weight") or name.endswith("norm.weight"):
                p.fill_(1.0)
            elif name.endswith(".bias"):
                p.normal_(0.0, std, generator=gen)
            else:
                p.normal_(0.0, std, generator=gen)

    def head_weight(self) -> torch.Tensor:
        return self.model.embed_tokens.weight if self.lm_head is None else self.lm_head.weight

    def _qkv(self, layer: _Layer, x: torch.Tensor):
        cfg = self.cfg
        b, t, _ = x.shape
        h = layer.input_layernorm(x)
        q = layer.self_attn.q_proj(h).view(b, t, cfg.num_attention_heads, cfg.head_dim)
        k = layer.self_attn.k_proj(h).view(b, t, cfg.num_key_value_heads, cfg.head_dim)
        v = layer.self_attn.v_proj(h).view(b, t, cfg.num_key_value_heads, cfg.head_dim)
        return q, k, v

    @torch.no_grad()
    def encode_chunks(self, chunks: torch.Tensor, lengths: torch.Tensor) -> LlamaChunkMemory:
        """Encode ``chunks`` ``[C, Tc]`` (each its own sequence, positions from 0, padded
        rows masked) into a ``LlamaChunkMemory``."""
        cfg = self.cfg
        c, tc = chunks.shape
        pos = torch.arange(tc, device=chunks.device).expand(c, tc)
        cos, sin = rope_tables(cfg, pos)
        valid = torch.arange(tc, device=chunks.device)[None] < lengths[:, None]
        x = self.model.embed_tokens(chunks).float()
        mem = LlamaChunkMemory(length=lengths.clone())
        for li, layer in enumerate(self.model.layers):
            q, k, v = self._qkv(layer, x)
            w = valid[:, :, None, None].float()
            mem.gist.append((k * w).sum(1).reshape(c, -1) / lengths.clamp_min(1)[:, None].float())
            qr, kr = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
            mem.k.append(kr)
            mem.v.append(v)
            a = self._attend(qr, kr, v, None, valid)
            x = self._finish_layer(layer, x, a)
        return mem

    def _attend(self, q, k, v, memory_kv, key_valid):
        """q ``[B,T,H,Dh]``, local k/v ``[B,T,Hkv,Dh]``; memory_kv: list per row of (k, v)
        ``[M, Hkv, Dh]`` or None.  One softmax over [memory ; causal local]."""
        cfg = self.cfg
        b, t, h, dh = q.shape
        g = cfg.group
        out = torch.empty_like(q)
        scale = 1.0 / math.sqrt(dh)
        causal = torch.ones(t, t, dtype=torch.bool, device=q.device).tril()
        for row in range(b):
            mk, mv = (memory_kv[row] if memory_kv is not None else (None, None))
            lk = k[row].repeat_interleave(g, dim=1)  # [T, H, Dh]
            lv = v[row].repeat_interleave(g, dim=1)
            mask = causal.clone()
            if key_valid is not None:
                mask &= key_valid[row][None, :]
            if mk is not None and mk.shape[0]:
                keys = torch.cat([mk.repeat_interleave(g, dim=1), lk], dim=0)
                vals = torch.cat([mv.repeat_interleave(g, dim=1), lv], dim=0)
                mask = torch.cat([torch.ones(t, mk.shape[0], dtype=torch.bool, device=q.device), mask], dim=1)
            else:
                keys, vals = lk, lv
            s = torch.einsum("thd,khd->htk", q[row], keys) * scale
            s = s.masked_fill(~mask[None], float("-inf"))
            p = torch.softmax(s, dim=-1).nan_to_num(0.0)
            out[row] = torch.einsum("htk,khd->thd", p, vals)
        return out

    def _finish_layer(self, layer, x, a):
        b, t = x.shape[:2]
        x = x + layer.self_attn.o_proj(a.reshape(b, t, -1))
        h = layer.post_attention_layernorm(x)
        m = layer.mlp
        return x + m.down_proj(F.silu(m.gate_proj(h)) * m.up_proj(h))

    @torch.no_grad()
    def forward(self, input_ids: torch.Tensor, attention_mask: torch.Tensor | None = None,
                memory: LlamaChunkMemory | None = None, return_selection: bool = False):
        """Logits ``[B, T, V]`` of a left-aligned prompt batch (positions 0..T-1), routed with
        the last valid token of each row."""
        cfg = self.cfg
        b, t = input_ids.shape
        pos = torch.arange(t, device=input_ids.device).expand(b, t)
        cos, sin = rope_tables(cfg, pos)
        valid = attention_mask.bool() if attention_mask is not None else None
        last = (valid.long().sum(1) - 1) if valid is not None else torch.full((b,), t - 1, device=input_ids.device)
        x = self.model.embed_tokens(input_ids).float()
        selections = []
        for li, layer in enumerate(self.model.layers):
            q, k, v = self._qkv(layer, x)
            memory_kv = None
            if memory is not None and cfg.is_pra_layer(li):
                route_q = q[torch.arange(b), last].view(b, cfg.num_key_value_heads, cfg.group, cfg.head_dim)
                picked = select_chunks(cfg, route_q.mean(2).reshape(b, -1), memory.gist[li], memory.namespace)
                selections.append(picked)
                memory_kv = []
                for row in range(b):
                    ks = [memory.k[li][c, : int(memory.length[c])] for c in picked[row]]
                    vs = [memory.v[li][c, : int(memory.length[c])] for c in picked[row]]
                    if ks:
                        memory_kv.append((torch.cat(ks), torch.cat(vs)))
                    else:
                        memory_kv.append((None, None))
            a = self._attend(apply_rope(q, cos, sin), apply_rope(k, cos, sin), v, memory_kv, valid)
            x = self._finish_layer(layer, x, a)
        logits = self.model.norm(x) @ self.head_weight().t()
        return (logits, selections) if return_selection else logits


@torch.no_grad()
def reference_step(model: PRALlamaReference, ids: torch.Tensor, cache: list, memory: LlamaChunkMemory | None,
                   namespace: list[int] | None, position_offset: int = 0):
    """Incremental fp32 step of ONE row: ``ids`` ``[T]`` continue the sequence whose per-layer
    post-rotary K/V are in ``cache`` (list of ``[k, v]`` ``[t, Hkv, Dh]``, extended in place).
    Routing uses the last new token; returns (logits ``[T, V]``, selections per PRA layer)."""
    cfg = model.cfg
    t0 = cache[0][0].shape[0] if cache and cache[0][0] is not None else 0
    T = ids.shape[0]
    pos = torch.arange(t0, t0 + T, device=ids.device)[None] + int(position_offset)
    cos, sin = rope_tables(cfg, pos)
    x = model.model.embed_tokens(ids[None]).float()
    picks = []
    scale = 1.0 / math.sqrt(cfg.head_dim)
    for li, layer in enumerate(model.model.layers):
        q, k, v = model._qkv(layer, x)
        keys_mem = vals_mem = None
        if memory is not None and namespace and cfg.is_pra_layer(li) and cfg.top_k_chunks > 0:
            rq = q[0, -1].view(cfg.num_key_value_heads, cfg.group, cfg.head_dim).mean(1).reshape(1, -1)
            sel = select_chunks(cfg, rq, memory.gist[li], [namespace])[0]
            picks.append(sel)
            if sel:
                keys_mem = torch.cat([memory.k[li][c, : int(memory.length[c])] for c in sel])
                vals_mem = torch.cat([memory.v[li][c, : int(memory.length[c])] for c in sel])
        qr, kr = apply_rope(q, cos, sin)[0], apply_rope(k, cos, sin)[0]
        if cache[li][0] is None:
            cache[li] = [kr, v[0]]
        else:
            cache[li] = [torch.cat([cache[li][0], kr]), torch.cat([cache[li][1], v[0]])]
        lk, lv = cache[li]
        n_loc = lk.shape[0]
        causal = torch.arange(n_loc, device=ids.device)[None, :] <= (t0 + torch.arange(T, device=ids.device))[:, None]
        if keys_mem is not None:
            keys, vals = torch.cat([keys_mem, lk]), torch.cat([vals_mem, lv])
            mask = torch.cat([torch.ones(T, keys_mem.shape[0], dtype=torch.bool, device=ids.device), causal], 1)
        else:
            keys, vals, mask = lk, lv, causal
        g = cfg.group
        s = torch.einsum("thd,khd->htk", qr, keys.repeat_interleave(g, 1)) * scale
        p = torch.softmax(s.masked_fill(~mask[None], float("-inf")), dim=-1)
        a = torch.einsum("htk,khd->thd", p, vals.repeat_interleave(g, 1))[None]
        x = model._finish_layer(layer, x, a)
    logits = (model.model.norm(x) @ model.head_weight().t())[0]
    return logits, picks


@torch.no_grad()
def reference_generate(model: PRALlamaReference, ids: torch.Tensor, length: int, memory, namespace,
                       max_new_tokens: int):
    """Greedy fp32 decoding of one row: prefill (routing with the last prompt token), then one
    token per step (routing with that token).  Returns (new ids, prefill logits of the last
    prompt token, selections of every step)."""
    cache = [[None, None] for _ in range(model.cfg.num_hidden_layers)]
    logits, picks = reference_step(model, ids[:length], cache, memory, namespace)
    first = logits[-1]
    steps = [picks]
    out = [int(first.argmax())]
    for _ in range(max_new_tokens - 1):
        logits, picks = reference_step(model, torch.tensor([out[-1]], device=ids.device), cache, memory, namespace)
        steps.append(picks)
        out.append(int(logits[-1].argmax()))
    return out, first, steps


def hf_config(cfg: PRALlamaConfig):
    """The matching Hugging Face config object (for loading weights / parity tests)."""
    import transformers

    common = dict(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size, intermediate_size=cfg.intermediate_size,
                  num_hidden_layers=cfg.num_hidden_layers, num_attention_heads=cfg.num_attention_heads,
                  num_key_value_heads=cfg.num_key_value_heads, rope_theta=cfg.rope_theta,
                  rms_norm_eps=cfg.rms_norm_eps, max_position_embeddings=cfg.max_position_embeddings,
                  tie_word_embeddings=cfg.tie_word_embeddings)
    if cfg.family == "qwen2":
        return transformers.Qwen2Config(**common)
    if cfg.family == "mistral":
        return transformers.MistralConfig(head_dim=cfg.head_dim, sliding_window=None, **common)
    return transformers.LlamaConfig(head_dim=cfg.head_dim, attention_bias=cfg.attention_bias, **common)
