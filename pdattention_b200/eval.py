"""``pra eval``: four prompt variants compared on the test split.

Variants (``src/pra_torch/eval.py:128-138`` defines the same four): the question
alone, the references' full texts prepended, their summaries prepended, and the
question with the references in PRA memory.  Each reports the LM loss over the
loader, the fraction of greedy generations containing the answer, the prompt's
token cost, and for the memory variant the reference / anchor / cache hits.  A
missing checkpoint gives a random-initialised model with a fitted character
tokenizer.
"""

from __future__ import annotations

import os
import time
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .config import PRAConfig
from .data.collators import PRACollator
from .data.tokenizer import BPETokenizer, PRATokenizer
from .memory.services import build_cache_from_metadata
from .models.tiny import TinyPRAModel
from .runtime.checkpointing import read_checkpoint

CharTokenizer = PRATokenizer


def build_training_corpus(examples) -> list[str]:
    """Texts a fitted character vocabulary must cover (question samples or core examples)."""
    texts = []
    for ex in examples:
        if hasattr(ex, "question"):
            texts.append(f"{ex.question} {ex.answer}")
            texts.extend(piece for ref in ex.references for piece in (ref.summary or "", str(ref.metadata.get("text", ""))))
        else:
            texts.extend([ex.prompt + ex.target, *ex.refs.values(), *ex.summaries.values()])
    return texts


@dataclass
class EvalResult:
    name: str
    exact: int
    total: int
    avg_input_tokens: float
    avg_resolved_refs: float
    answer_exact_match: float
    expected_ref_hit: float
    expected_anchor_hit: float
    avg_num_expansions: float
    avg_retrieved_tokens: float
    avg_full_context_tokens: float
    lm_loss: float
    cache_hit_ratio: float
    latency: float
    sample_output: str

    @property
    def accuracy(self) -> float:
        return self.exact / max(self.total, 1)


def load_model_and_tokenizer(ckpt_path: str, device: str, examples, *, max_seq_len: int = 96, d_model: int = 128,
                             n_heads: int = 4, n_layers: int = 4, n_vanilla_layers: int = 0, n_mixed_layers: int = 0,
                             dropout: float = 0.0, pra_layer_ids=(2, 3), top_k_references: int = 2,
                             top_k_chunks_per_reference: int = 1, trigger_threshold: float = 0.2,
                             memory_transport: str = "native_kv", use_cross_attention_memory=None,
                             use_concat_memory=None, memory_alpha: float = 0.5, resolver_config=None,
                             cache_config=None, **routing_kwargs):
    """Restore (or randomly initialise) a model and its tokenizer; returns ``(model, tokenizer, loaded)``.

    A checkpoint restores ``PRAConfig(**cfg)`` with ``device`` overridden and its BPE or character
    tokenizer; without one, a character tokenizer is fitted to ``examples`` and the model is built
    from the keyword arguments."""
    if os.path.exists(ckpt_path):
        checkpoint = read_checkpoint(ckpt_path, map_location=device)
        cfg = PRAConfig(**{**dict(checkpoint["cfg"]), "device": device})
        bpe = checkpoint.get("tokenizer_type") == "BPETokenizer" and checkpoint.get("tokenizer_json")
        tokenizer = BPETokenizer.from_json(checkpoint["tokenizer_json"]) if bpe else \
            CharTokenizer.from_vocab(checkpoint["stoi"])
        model = TinyPRAModel(cfg).to(device)
        model.load_state_dict(checkpoint["model"])
        return model.eval(), tokenizer, True
    tokenizer = CharTokenizer(build_training_corpus(examples))
    cfg = PRAConfig(vocab_size=tokenizer.vocab_size, d_model=d_model, n_heads=n_heads, n_layers=n_layers,
                    n_vanilla_layers=n_vanilla_layers, n_mixed_layers=n_mixed_layers, max_seq_len=max_seq_len,
                    dropout=dropout, pra_layer_ids=tuple(pra_layer_ids), top_k_references=top_k_references,
                    top_k_chunks_per_reference=top_k_chunks_per_reference, trigger_threshold=trigger_threshold,
                    memory_transport=memory_transport, use_cross_attention_memory=use_cross_attention_memory,
                    use_concat_memory=use_concat_memory, memory_alpha=memory_alpha, device=device, **routing_kwargs)
    return TinyPRAModel(cfg).to(device), tokenizer, False


def generate_greedy(model, tokenizer, prompt: str, device: str, max_new_tokens: int) -> str:
    """Greedy continuation without memory (the prompt window slides at ``max_seq_len``)."""
    ids = torch.tensor([tokenizer.encode(prompt)], dtype=torch.long, device=device)
    window = model.cfg.max_seq_len
    for _ in range(max_new_tokens):
        nxt = model(ids[:, -window:], use_pra_memory=False)[:, -1].argmax(dim=-1, keepdim=True)
        ids = torch.cat([ids, nxt], dim=1)
    return tokenizer.decode(ids[0])


def generate_pra(model, tokenizer, prompt: str, device: str, max_new_tokens: int) -> str:
    """Greedy continuation through the model's PRA memory (its attached cache)."""
    ids = torch.tensor([tokenizer.encode(prompt)], dtype=torch.long, device=device)
    return tokenizer.decode(model.generate(ids, max_new_tokens=max_new_tokens, tokenizer=tokenizer, do_sample=False)[0])


# The four compared prompts: the question alone, every reference's full text in front of it,
# the reference summaries in front of it (a retrieval-by-summary stand-in), and the question
# alone with the references in PRA memory.
def _prompt_set(question: str, texts: list[str], summaries: list[str]) -> dict:
    return {"no_refs": question, "full_context": "Context:\n" + "\n".join(texts) + "\n\n" + question,
            "simple_rag": "Retrieved summary:\n" + "\n".join(summaries) + "\n\n" + question, "pra": question}


def baseline_prompts_from_metadata(item) -> dict:
    refs = item["references"]
    return _prompt_set(item["question"], [str(r.metadata.get("text", "")) for r in refs],
                       [r.summary or "" for r in refs])


def baseline_prompts(ex) -> dict:
    if hasattr(ex, "references"):
        return baseline_prompts_from_metadata({"question": ex.question, "references": ex.references})
    return _prompt_set(ex.prompt, list(ex.refs.values()), list(ex.summaries.values()))


def generated_contains_target(output: str, prompt: str, target: str) -> bool:
    return target.strip() in output[len(prompt):]


class _Tally:
    """Running sums of one variant's evaluation."""

    def __init__(self):
        self.n = self.exact = self.ref_hits = self.anchor_hits = 0
        self.input_tokens = self.full_tokens = self.resolved = self.retrieved = 0
        self.losses: list[float] = []
        self.sample = ""

    def per_example(self, value) -> float:
        return value / max(self.n, 1)


def _memory_hits(cache, item) -> tuple[bool, bool]:
    """(every expected reference is cached, an expected anchor appears in the cached texts or URIs)."""
    expected = {r.uri for r in item["references"] if r.id in item["target_reference_ids"]}
    ref_hit = not expected or bool(expected.intersection(cache.entries))
    anchors = item.get("expected_anchors", [])
    texts, uris = "\n".join(e.text for e in cache.all_entries()), " ".join(cache.entries)
    return ref_hit, not anchors or any(a in texts or a in uris for a in anchors)


def evaluate_variant(name, model, tokenizer, dataloader, device, max_new_tokens, *, resolver_config=None,
                     cache_config=None) -> EvalResult:
    """LM loss over the loader and greedy-generation accuracy of one prompt variant."""
    started = time.perf_counter()
    with_memory = name == "pra"
    tally = _Tally()
    for batch in dataloader:
        ids, labels = batch["input_ids"].to(device), batch["labels"].to(device)
        if with_memory:
            cache = build_cache_from_metadata(model, tokenizer, batch["metadata"], device,
                                              resolver_config=resolver_config, cache_config=cache_config)
            tally.resolved += len(cache.entries)
            tally.retrieved += sum(len(tokenizer.encode(e.text)) for e in cache.all_entries())
            logits = model(ids)
        else:
            model.clear_pra_cache()
            logits = model(ids, use_pra_memory=False)
        tally.losses.append(float(F.cross_entropy(logits.flatten(0, 1), labels.flatten(), ignore_index=0).detach().cpu()))
        for item in batch["metadata"]:
            prompts = baseline_prompts_from_metadata(item)
            prompt = prompts[name]
            tally.input_tokens += len(tokenizer.encode(prompt))
            tally.full_tokens += len(tokenizer.encode(prompts["full_context"]))
            if with_memory:
                ref_hit, anchor_hit = _memory_hits(model.pra_cache, item)
                tally.ref_hits += ref_hit
                tally.anchor_hits += anchor_hit
            generate = generate_pra if with_memory else generate_greedy
            output = generate(model, tokenizer, prompt, device, max_new_tokens)
            tally.exact += generated_contains_target(output, prompt, item["answer"].strip())
            tally.sample = tally.sample if tally.n else output
            tally.n += 1
    hit = (lambda v: tally.per_example(v)) if with_memory else (lambda v: 0.0)
    return EvalResult(name, tally.exact, tally.n, tally.per_example(tally.input_tokens),
                      tally.per_example(tally.resolved), tally.per_example(tally.exact), hit(tally.ref_hits),
                      hit(tally.anchor_hits), 0.0, tally.per_example(tally.retrieved),
                      tally.per_example(tally.full_tokens), sum(tally.losses) / max(len(tally.losses), 1),
                      hit(tally.ref_hits), time.perf_counter() - started, tally.sample)


_REPORT_HEADER = ("variant       loss     accuracy   input_tokens   resolved_refs   ref_hit   anchor_hit   cache_hit"
                  "   latency")


def print_report(results, loaded_checkpoint: bool) -> None:
    print(f"PRA eval report ({'checkpoint' if loaded_checkpoint else 'random initialization'})")
    print(_REPORT_HEADER)
    for r in results:
        print(f"{r.name:<13} {r.lm_loss:>6.3f} {r.accuracy:>7.2%} {r.avg_input_tokens:>14.1f} "
              f"{r.avg_resolved_refs:>15.1f} {r.expected_ref_hit:>8.2%} {r.expected_anchor_hit:>11.2%} "
              f"{r.cache_hit_ratio:>10.2%} {r.latency:>8.3f}s")
    print("\nSample PRA output:")
    for r in results:
        if r.name == "pra":
            print(r.sample_output)
            break


VARIANTS = ("no_refs", "full_context", "simple_rag", "pra")


def run_evaluation(*, ckpt: str, device: str, datamodule, max_new_tokens: int, max_seq_len: int = 96,
                   resolver_config=None, cache_config=None, **model_kwargs):
    """Restore the model (or initialise one), rebuild the data module's collator for its tokenizer
    and evaluate every variant on the test split."""
    model, tokenizer, loaded = load_model_and_tokenizer(ckpt, device, datamodule.dataset, max_seq_len=max_seq_len,
                                                        **model_kwargs)
    datamodule.tokenizer = tokenizer
    datamodule.collator = PRACollator(tokenizer, max_seq_len=max_seq_len)
    results = [evaluate_variant(name, model, tokenizer, datamodule.test_loader(), device, max_new_tokens,
                                resolver_config=resolver_config, cache_config=cache_config) for name in VARIANTS]
    print_report(results, loaded)
    return results
