"""``pra eval``: compare no_refs / full_context / simple_rag / pra on the test split.

Behaviour of ``src/pra_torch/eval.py``: a missing checkpoint falls back to a
random-initialised model with a corpus-built character tokenizer; a checkpoint
restores ``PRAConfig(**cfg)`` (device overridden) and a BPE or character
tokenizer; every variant reports LM loss, containment accuracy of greedy
generations, input-token cost and (for pra) reference / anchor / cache hits.
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
    texts = []
    for ex in examples:
        if hasattr(ex, "question"):
            texts.append(ex.question + " " + ex.answer)
            for ref in ex.references:
                texts += [ref.summary or "", str(ref.metadata.get("text", ""))]
        else:
            texts.append(ex.prompt + ex.target)
            texts += list(ex.refs.values()) + list(ex.summaries.values())
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
    """Restore (or randomly initialise) a model and its tokenizer; returns ``(model, tokenizer, loaded)``."""
    if not os.path.exists(ckpt_path):
        tokenizer = CharTokenizer(build_training_corpus(examples))
        cfg = PRAConfig(vocab_size=tokenizer.vocab_size, d_model=d_model, n_heads=n_heads, n_layers=n_layers,
                        n_vanilla_layers=n_vanilla_layers, n_mixed_layers=n_mixed_layers, max_seq_len=max_seq_len,
                        dropout=dropout, pra_layer_ids=tuple(pra_layer_ids), top_k_references=top_k_references,
                        top_k_chunks_per_reference=top_k_chunks_per_reference, trigger_threshold=trigger_threshold,
                        memory_transport=memory_transport, use_cross_attention_memory=use_cross_attention_memory,
                        use_concat_memory=use_concat_memory, memory_alpha=memory_alpha, device=device,
                        **routing_kwargs)
        return TinyPRAModel(cfg).to(device), tokenizer, False
    checkpoint = read_checkpoint(ckpt_path, map_location=device)
    values = dict(checkpoint["cfg"])
    values["device"] = device
    cfg = PRAConfig(**values)
    if checkpoint.get("tokenizer_type") == "BPETokenizer" and checkpoint.get("tokenizer_json"):
        tokenizer = BPETokenizer.from_json(checkpoint["tokenizer_json"])
    else:
        tokenizer = CharTokenizer.from_vocab(checkpoint["stoi"])
    model = TinyPRAModel(cfg).to(device)
    model.load_state_dict(checkpoint["model"])
    model.eval()
    return model, tokenizer, True


def generate_greedy(model, tokenizer, prompt: str, device: str, max_new_tokens: int) -> str:
    ids = torch.tensor([tokenizer.encode(prompt)], dtype=torch.long, device=device)
    for _ in range(max_new_tokens):
        logits = model(ids[:, -model.cfg.max_seq_len:], use_pra_memory=False)
        ids = torch.cat([ids, logits[:, -1, :].argmax(dim=-1, keepdim=True)], dim=1)
    return tokenizer.decode(ids[0])


def generate_pra(model, tokenizer, prompt: str, device: str, max_new_tokens: int) -> str:
    ids = torch.tensor([tokenizer.encode(prompt)], dtype=torch.long, device=device)
    out = model.generate(ids, max_new_tokens=max_new_tokens, tokenizer=tokenizer, do_sample=False)
    return tokenizer.decode(out[0])


def baseline_prompts_from_metadata(item) -> dict:
    refs, question = item["references"], item["question"]
    docs = "\n".join(str(r.metadata.get("text", "")) for r in refs)
    summaries = "\n".join(r.summary or "" for r in refs)
    return {"no_refs": question, "full_context": f"Context:\n{docs}\n\n{question}",
            "simple_rag": f"Retrieved summary:\n{summaries}\n\n{question}", "pra": question}


def baseline_prompts(ex) -> dict:
    if hasattr(ex, "references"):
        return baseline_prompts_from_metadata({"question": ex.question, "references": ex.references})
    docs, summaries = "\n".join(ex.refs.values()), "\n".join(ex.summaries.values())
    return {"no_refs": ex.prompt, "full_context": f"Context:\n{docs}\n\n{ex.prompt}",
            "simple_rag": f"Retrieved summary:\n{summaries}\n\n{ex.prompt}", "pra": ex.prompt}


def generated_contains_target(output: str, prompt: str, target: str) -> bool:
    return target.strip() in output[len(prompt):]


def evaluate_variant(name, model, tokenizer, dataloader, device, max_new_tokens, *, resolver_config=None,
                     cache_config=None) -> EvalResult:
    t0 = time.perf_counter()
    exact = ref_hits = anchor_hits = cache_hits = cost = resolved = retrieved = full_cost = total = 0
    loss_sum, loss_count, sample = 0.0, 0, ""
    for batch in dataloader:
        ids, labels = batch["input_ids"].to(device), batch["labels"].to(device)
        if name == "pra":
            cache = build_cache_from_metadata(model, tokenizer, batch["metadata"], device,
                                              resolver_config=resolver_config, cache_config=cache_config)
            resolved += len(cache.entries)
            retrieved += sum(len(tokenizer.encode(e.text)) for e in cache.all_entries())
            logits = model(ids)
        else:
            model.clear_pra_cache()
            logits = model(ids, use_pra_memory=False)
        loss_sum += float(F.cross_entropy(logits.view(-1, logits.size(-1)), labels.view(-1), ignore_index=0).detach().cpu())
        loss_count += 1
        for item in batch["metadata"]:
            prompts = baseline_prompts_from_metadata(item)
            prompt, target = prompts[name], item["answer"].strip()
            cost += len(tokenizer.encode(prompt))
            full_cost += len(tokenizer.encode(prompts["full_context"]))
            if name == "pra":
                expected = {r.uri for r in item["references"] if r.id in item["target_reference_ids"]}
                if not expected or expected.intersection(model.pra_cache.entries):
                    ref_hits += 1
                    cache_hits += 1
                anchors = item.get("expected_anchors", [])
                text = "\n".join(e.text for e in model.pra_cache.all_entries())
                if not anchors or any(a in text or a in " ".join(model.pra_cache.entries) for a in anchors):
                    anchor_hits += 1
                output = generate_pra(model, tokenizer, prompt, device, max_new_tokens)
            else:
                output = generate_greedy(model, tokenizer, prompt, device, max_new_tokens)
            exact += int(generated_contains_target(output, prompt, target))
            sample = output if total == 0 else sample
            total += 1
    n = max(total, 1)
    pra = name == "pra"
    return EvalResult(name, exact, total, cost / n, resolved / n, exact / n, ref_hits / n if pra else 0.0,
                      anchor_hits / n if pra else 0.0, 0.0, retrieved / n, full_cost / n,
                      loss_sum / max(loss_count, 1), cache_hits / n if pra else 0.0, time.perf_counter() - t0, sample)


def print_report(results, loaded_checkpoint: bool) -> None:
    print(f"PRA eval report ({'checkpoint' if loaded_checkpoint else 'random initialization'})")
    print("variant       loss     accuracy   input_tokens   resolved_refs   ref_hit   anchor_hit   cache_hit   latency")
    for r in results:
        print(f"{r.name:<13} {r.lm_loss:>6.3f} {r.accuracy:>7.2%} {r.avg_input_tokens:>14.1f} "
              f"{r.avg_resolved_refs:>15.1f} {r.expected_ref_hit:>8.2%} {r.expected_anchor_hit:>11.2%} "
              f"{r.cache_hit_ratio:>10.2%} {r.latency:>8.3f}s")
    print("\nSample PRA output:")
    pra = next((r for r in results if r.name == "pra"), None)
    if pra is not None:
        print(pra.sample_output)


def run_evaluation(*, ckpt: str, device: str, datamodule, max_new_tokens: int, max_seq_len: int = 96,
                   resolver_config=None, cache_config=None, **model_kwargs):
    model, tokenizer, loaded = load_model_and_tokenizer(ckpt, device, datamodule.dataset, max_seq_len=max_seq_len,
                                                        **model_kwargs)
    datamodule.tokenizer = tokenizer
    datamodule.collator = PRACollator(tokenizer, max_seq_len=max_seq_len)
    results = [evaluate_variant(name, model, tokenizer, datamodule.test_loader(), device, max_new_tokens,
                                resolver_config=resolver_config, cache_config=cache_config)
               for name in ("no_refs", "full_context", "simple_rag", "pra")]
    print_report(results, loaded)
    return results
