"""A tiny end-to-end TinyGPT-PRA training step used by the smoke check and GPU tests.

The model has head width 64 (d_model 128, 2 heads), so the step runs the
tcgen05/TMEM attention kernels (forward, packed short-sequence forward, dQ and
dK/dV) rather than the mma.sync ones kept for head width 32.
"""

from __future__ import annotations

import tempfile
from pathlib import Path

import torch

from .config import PRAConfig, ResolverServiceConfig
from .data import PRADataModule, WordIdTokenizer
from .data.generators import generate_hierarchical_tokens
from .models.fastpath import prepare_model
from .pra_train import _pra_batch_step


def tiny_config(vocab: int) -> PRAConfig:
    return PRAConfig(vocab_size=vocab, d_model=128, n_heads=2, n_layers=2, max_seq_len=256, model_variant="td_pra",
                     chunking_mode="fixed", fixed_chunk_tokens=32, top_k_references=2, top_k_chunks_per_reference=2,
                     gist_mode="kmeans", gists_per_chunk=2, recursive_refs_enabled=True, trigger_threshold=-1.0,
                     device="cuda")


def tiny_batch(root: Path, vocab: int = 500, examples: int = 4):
    generate_hierarchical_tokens(root / "synthetic_hierarchical_tokens", examples=examples, doc_tokens=48,
                                 prompt_tokens=95, vocab=vocab, roots=2, children=1, grandchildren=2)
    tok = WordIdTokenizer(vocab)
    dm = PRADataModule("synthetic_hierarchical_tokens", str(root), batch_size=examples, max_seq_len=256,
                       tokenizer=tok, shuffle=False).load()
    return tok, next(iter(dm._loader(dm.dataset, shuffle=False)))


def tiny_training_step(device) -> float:
    torch.manual_seed(0)
    with tempfile.TemporaryDirectory() as tmp:
        tok, batch = tiny_batch(Path(tmp))
        model = prepare_model(tiny_config(tok.vocab_size), device)
        assert getattr(model, "_device_runtime", None) is not None, "device path not attached"
        from .config import TrainConfig

        opt = model.build_optimizer(TrainConfig(device=str(device)))
        loss, _ = _pra_batch_step(model, batch, str(device), tok, ResolverServiceConfig(), None)
        loss.backward()
        opt.step()
        torch.cuda.synchronize(device)
        return float(loss.item())
