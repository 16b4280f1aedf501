"""Plain causal-LM training and evaluation without PRA memory (the LM adapter).

Same entry points and metrics as ``src/pra_torch/lm_train.py:16-82``: token-level
loss (pad id 0 included, as the LM blocks carry no padding), perplexity, token
accuracy and throughput; checkpoints carry the model config and tokenizer.
"""

from __future__ import annotations

import time

import torch
import torch.nn.functional as F

from .models.tiny import TinyPRAModel
from .runtime.metrics import cuda_memory_allocated, perplexity
from .runtime.train import create_training_state, default_batch_step, move_batch, train_model


@torch.no_grad()
def _score_batch(model, batch) -> tuple[float, int, int]:
    """(summed loss, tokens, correct next-token predictions) of one batch."""
    logits = model(batch["input_ids"], use_pra_memory=False).flatten(0, 1)
    labels = batch["labels"].flatten()
    loss = F.cross_entropy(logits, labels, reduction="sum")
    return float(loss.cpu()), int(labels.numel()), int((logits.argmax(dim=-1) == labels).sum())


def evaluate_language_model(*, model, loader, device: str, split: str = "val") -> dict:
    restore = model.training
    model.eval()
    started = time.perf_counter()
    totals = [0.0, 0, 0]
    for batch in loader:
        for i, value in enumerate(_score_batch(model, move_batch(batch, device))):
            totals[i] += value
    model.train(restore)
    loss_sum, tokens, correct = totals
    elapsed = max(time.perf_counter() - started, 1e-9)
    loss = loss_sum / max(tokens, 1)
    return {f"{split}_loss": loss, "loss": loss, "perplexity": perplexity(loss),
            "token_accuracy": correct / max(tokens, 1), "tokens": tokens, "tokens_per_second": tokens / elapsed,
            "latency": elapsed, "gpu_memory_allocated": cuda_memory_allocated(device)}


def train_language_model(*, cfg, train_config, datamodule, model=None):
    tokenizer = datamodule.tokenizer

    def checkpoint_extra() -> dict:
        return {"cfg": cfg.__dict__, "stoi": tokenizer.stoi, "itos": tokenizer.itos,
                "tokenizer_type": type(tokenizer).__name__,
                "tokenizer_json": tokenizer.to_json() if hasattr(tokenizer, "to_json") else None,
                "dataset_stage": train_config.dataset_stage}

    state = create_training_state(model or TinyPRAModel(cfg), train_config, checkpoint_extra=checkpoint_extra)
    return train_model(model=state.model, train_config=train_config, train_loader=datamodule.train_loader(),
                       val_loader=datamodule.val_loader(), test_loader=datamodule.test_loader(),
                       batch_step=lambda m, b, d: default_batch_step(m, b, d, ignore_index=0),
                       eval_step=lambda m, loader, d, split="val": evaluate_language_model(
                           model=m, loader=loader, device=d, split=split),
                       state=state)
