"""Plain causal-LM training without memory (``src/pra_torch/lm_train.py``)."""

from __future__ import annotations

import time

import torch
import torch.nn.functional as F

from .models.tiny import TinyPRAModel
from .runtime.metrics import cuda_memory_allocated, perplexity
from .runtime.train import create_training_state, default_batch_step, move_batch, train_model


def evaluate_language_model(*, model, loader, device: str, split: str = "val") -> dict:
    was_training = model.training
    model.eval()
    loss_sum = tokens = correct = 0
    t0 = time.perf_counter()
    with torch.no_grad():
        for batch in loader:
            batch = move_batch(batch, device)
            logits = model(batch["input_ids"], use_pra_memory=False)
            labels = batch["labels"].reshape(-1)
            n = int(labels.numel())
            loss_sum += float(F.cross_entropy(logits.reshape(-1, logits.size(-1)), labels).cpu()) * n
            tokens += n
            correct += int((logits.argmax(dim=-1).reshape(-1) == labels).sum().item())
    if was_training:
        model.train()
    elapsed = max(time.perf_counter() - t0, 1e-9)
    loss = loss_sum / max(tokens, 1)
    return {f"{split}_loss": loss, "loss": loss, "perplexity": perplexity(loss),
            "token_accuracy": correct / max(tokens, 1), "tokens": tokens, "tokens_per_second": tokens / elapsed,
            "latency": elapsed, "gpu_memory_allocated": cuda_memory_allocated(device)}


def train_language_model(*, cfg, train_config, datamodule, model=None):
    tokenizer = datamodule.tokenizer
    model = model or TinyPRAModel(cfg)
    extra = lambda: {"cfg": cfg.__dict__, "stoi": tokenizer.stoi, "itos": tokenizer.itos,  # noqa: E731
                     "tokenizer_type": type(tokenizer).__name__,
                     "tokenizer_json": tokenizer.to_json() if hasattr(tokenizer, "to_json") else None,
                     "dataset_stage": train_config.dataset_stage}
    state = create_training_state(model, train_config, checkpoint_extra=extra)
    return train_model(model=state.model, train_config=train_config, train_loader=datamodule.train_loader(),
                       val_loader=datamodule.val_loader(), test_loader=datamodule.test_loader(),
                       batch_step=lambda m, b, d: default_batch_step(m, b, d, ignore_index=0),
                       eval_step=lambda m, loader, d, split="val": evaluate_language_model(model=m, loader=loader,
                                                                                            device=d, split=split),
                       state=state)
