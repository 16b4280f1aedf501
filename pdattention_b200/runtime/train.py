"""Generic training engine (one canonical loop with injected batch / eval steps).

Contract of ``src/common/train.py:24-486``: AdamW + linear-warmup ``LambdaLR``,
gradient accumulation, clip + grad-norm + scheduler per optimizer step,
validation / checkpoint cadence by optimizer step, ``latest.pt`` / ``best.pt``
payloads (model, optimizer, scheduler, config, counters + extras), end-of-epoch
validation, final test and run timing metrics.

B200 additions:

* a model may provide ``optimizer_step_hook`` (the fused-AdamW + fused DP
  reduction path of ``pdattention_b200.parallel.engine``) which replaces the
  stock clip/step sequence;
* batch timing uses CUDA events instead of a host synchronise around every
  batch (``sync_every_batch=True`` restores the reference behaviour);
* checkpoints and loggers are rank-0 only under ``torch.distributed``.
"""

from __future__ import annotations

import random
import time
from contextlib import nullcontext
from dataclasses import dataclass, field
from pathlib import Path
from typing import Callable

import numpy as np
import torch
import torch.nn.functional as F

from .callbacks import EarlyStopping, ModelCheckpoint
from .checkpointing import atomic_save, load_checkpoint, serializable_config
from .logging import build_logger
from .metrics import DeviceTimer, RunningAverages, cuda_memory_allocated, grad_norm, perplexity


_END = object()  # end-of-loader sentinel for the one-batch lookahead


def _rank() -> int:
    if torch.distributed.is_available() and torch.distributed.is_initialized():
        return torch.distributed.get_rank()
    return 0


@dataclass
class TrainingState:
    model: torch.nn.Module
    train_config: object
    device: str
    optimizer: torch.optim.Optimizer
    scheduler: object
    run_dir: Path
    checkpoint: ModelCheckpoint
    logger: object
    scaler: object | None
    early_stopping: EarlyStopping
    global_step: int = 0
    batch_step: int = 0
    start_epoch: int = 0
    best_val_loss: float = float("inf")
    epoch_history: list[dict] = field(default_factory=list)
    checkpoint_extra: Callable[[], dict] | None = None
    logger_closed: bool = False


def resolve_device(device: str) -> str:
    if device == "auto":
        return "cuda" if torch.cuda.is_available() else "cpu"
    return device


def seed_everything(seed: int) -> None:
    random.seed(seed)
    np.random.seed(seed)
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)


def move_batch(batch, device: str, non_blocking: bool = False):
    if torch.is_tensor(batch):
        return batch.to(device, non_blocking=non_blocking)
    if isinstance(batch, dict):
        return {k: move_batch(v, device, non_blocking) for k, v in batch.items()}
    if isinstance(batch, list):
        return [move_batch(v, device, non_blocking) for v in batch]
    if isinstance(batch, tuple):
        return tuple(move_batch(v, device, non_blocking) for v in batch)
    return batch


def warmup_lambda(warmup_steps: int):
    def factor(step: int) -> float:
        if warmup_steps and step < warmup_steps:
            return max(step, 1) / warmup_steps
        return 1.0

    return factor


def create_training_state(model, train_config, *, optimizer=None, scheduler=None,
                          checkpoint_extra: Callable[[], dict] | None = None) -> TrainingState:
    seed_everything(train_config.seed)
    device = resolve_device(train_config.device)
    model.to(device)
    broadcast_parameters(model)  # data parallel: every rank starts from rank 0's weights
    sync = getattr(model, "after_load_state", None)
    if sync is not None:
        sync()
    build_optimizer = getattr(model, "build_optimizer", None)
    if optimizer is None:
        optimizer = (build_optimizer(train_config) if build_optimizer is not None else
                     torch.optim.AdamW(model.parameters(), lr=train_config.learning_rate,
                                       weight_decay=train_config.weight_decay))
        world = torch.distributed.get_world_size() if (torch.distributed.is_available() and
                                                       torch.distributed.is_initialized()) else 1
        if world > 1 and getattr(model, "_device_runtime", None) is not None:
            from ..parallel.dp import attach_data_parallel

            # fused peer-memory gradient average; overlapped with the backward unless micro-batches
            # accumulate (a block's gradient is final only after the last micro-batch)
            attach_data_parallel(model, optimizer, world,
                                 overlap=False if int(train_config.grad_accum_steps) > 1 else None)
    if scheduler is None:
        scheduler = torch.optim.lr_scheduler.LambdaLR(optimizer, warmup_lambda(train_config.warmup_steps))
    run_dir = Path(train_config.output_dir) / train_config.experiment_name
    rank = _rank()
    checkpoint = ModelCheckpoint(run_dir / "checkpoints")
    logger = build_logger(train_config, run_dir, rank=rank)
    logger.log_config(train_config)
    use_scaler = train_config.mixed_precision and device.startswith("cuda") and not getattr(model, "bf16_native", False)
    state = TrainingState(model=model, train_config=train_config, device=device, optimizer=optimizer,
                          scheduler=scheduler, run_dir=run_dir, checkpoint=checkpoint, logger=logger,
                          scaler=torch.amp.GradScaler("cuda") if use_scaler else None,
                          early_stopping=EarlyStopping(train_config.early_stopping_patience),
                          checkpoint_extra=checkpoint_extra)
    if train_config.resume_from:
        resume_training_state(state, train_config.resume_from)
    return state


def resume_training_state(state: TrainingState, path) -> dict:
    checkpoint = load_checkpoint(path, state.model, state.optimizer, state.scheduler, map_location=state.device)
    state.start_epoch = int(checkpoint.get("epoch", 0))
    state.global_step = int(checkpoint.get("global_step", 0))
    state.batch_step = int(checkpoint.get("batch_step", state.global_step))
    state.best_val_loss = float(checkpoint.get("best_val_loss", float("inf")))
    state.early_stopping.best = state.best_val_loss
    sync = getattr(state.model, "after_load_state", None)
    if sync is not None:
        sync()
    return checkpoint


def save_training_state(state: TrainingState, path, epoch: int) -> Path:
    path = Path(path)
    if _rank() != 0:
        return path
    payload = {
        "model": state.model.state_dict(),
        "optimizer": state.optimizer.state_dict(),
        "scheduler": state.scheduler.state_dict() if state.scheduler is not None else None,
        "config": serializable_config(state.train_config),
        "epoch": epoch,
        "global_step": state.global_step,
        "batch_step": state.batch_step,
        "best_val_loss": state.best_val_loss,
    }
    if state.checkpoint_extra:
        payload.update(state.checkpoint_extra())
    return atomic_save(payload, path)


def close_training_state(state: TrainingState) -> None:
    if not state.logger_closed:
        state.logger.close()
        state.logger_closed = True


def default_batch_step(model, batch: dict, device: str, *, ignore_index: int = -100):
    batch = move_batch(batch, device)
    logits = model(batch["input_ids"])
    logits = getattr(logits, "logits", logits)
    loss = F.cross_entropy(logits.reshape(-1, logits.size(-1)), batch["labels"].reshape(-1), ignore_index=ignore_index)
    mask = batch.get("attention_mask")
    tokens = int(mask.sum().item()) if mask is not None else int((batch["labels"] != ignore_index).sum().item())
    return loss, {"tokens": tokens, "examples": int(batch["input_ids"].shape[0])}


def validated_extra_metrics(values: dict | None, reserved: set[str]) -> dict[str, float]:
    out = {}
    for key, value in (values or {}).items():
        if key in reserved or not isinstance(key, str):
            continue
        if torch.is_tensor(value):
            if value.numel() != 1:
                continue
            value = value.detach().item()
        if isinstance(value, (int, float, bool)):
            out[key] = float(value)
    return out


def _validation_checkpoint(state: TrainingState, metrics: dict, epoch: int) -> bool:
    val_loss = metrics.get("val_loss", metrics.get("loss", float("inf")))
    improved = val_loss < state.best_val_loss
    if improved:
        state.best_val_loss = val_loss
    save_training_state(state, state.checkpoint.latest_path, epoch)
    if improved:
        save_training_state(state, state.checkpoint.best_path, epoch)
    return state.early_stopping.update(val_loss)


def average_gradients(model) -> None:
    """Data parallel: every rank's gradients become the mean over ranks (one flat all-reduce;
    gloo on CPU, NCCL on GPU).  No-op outside a process group."""
    if not (torch.distributed.is_available() and torch.distributed.is_initialized()):
        return
    world = torch.distributed.get_world_size()
    if world <= 1:
        return
    grads = [p.grad for p in model.parameters() if p.grad is not None]
    if not grads:
        return
    flat = torch.cat([g.reshape(-1).float() for g in grads])
    torch.distributed.all_reduce(flat, op=torch.distributed.ReduceOp.SUM)
    flat /= world
    offset = 0
    for g in grads:
        g.copy_(flat[offset: offset + g.numel()].view_as(g))
        offset += g.numel()


def broadcast_parameters(model, src: int = 0) -> None:
    """Start every data-parallel rank from rank ``src``'s parameters."""
    if not (torch.distributed.is_available() and torch.distributed.is_initialized()):
        return
    if torch.distributed.get_world_size() <= 1:
        return
    with torch.no_grad():
        for p in model.parameters():
            torch.distributed.broadcast(p.data, src=src)


def _stock_optimizer_step(state: TrainingState, model, train_config) -> float:
    optimizer = state.optimizer
    average_gradients(model)
    if state.scaler is not None:
        state.scaler.unscale_(optimizer)
    norm = grad_norm(model.parameters())
    if train_config.max_grad_norm:
        torch.nn.utils.clip_grad_norm_(model.parameters(), train_config.max_grad_norm)
    if state.scaler is not None:
        state.scaler.step(optimizer)
        state.scaler.update()
    else:
        optimizer.step()
    return norm


def train_model(*, model, train_config, train_loader, val_loader=None, test_loader=None, optimizer=None,
                scheduler=None, batch_step=default_batch_step, eval_step=None, checkpoint_extra=None,
                state: TrainingState | None = None, sync_every_batch: bool | None = None):
    """Run epochs of ``batch_step`` + backward + optimizer updates with eval/checkpoint cadence."""
    run_start = time.perf_counter()
    state = state or create_training_state(model, train_config, optimizer=optimizer, scheduler=scheduler,
                                           checkpoint_extra=checkpoint_extra)
    if checkpoint_extra is not None:
        state.checkpoint_extra = checkpoint_extra
    model, optimizer, scheduler = state.model, state.optimizer, state.scheduler
    hook = getattr(model, "optimizer_step_hook", None)
    if sync_every_batch is None:
        sync_every_batch = hook is None
    cuda = state.device.startswith("cuda") and torch.cuda.is_available()

    def synchronize():
        if cuda:
            torch.cuda.synchronize()

    def timed_evaluation(loader, split: str):
        synchronize()
        t0 = time.perf_counter()
        values = eval_step(model, loader, state.device, split=split)
        synchronize()
        values[f"{split}_duration_seconds"] = max(time.perf_counter() - t0, 1e-9)
        return values, values[f"{split}_duration_seconds"]

    last_val: dict = {}
    epoch_metrics: dict = {}
    stop = bool(train_config.max_steps is not None and state.global_step >= train_config.max_steps)
    last_epoch = state.start_epoch
    last_val_step = -1
    train_s = val_s = test_s = 0.0
    processed_tokens = sequences = 0
    accum = max(int(train_config.grad_accum_steps), 1)

    for epoch in range(state.start_epoch, train_config.epochs):
        if stop:
            break
        last_epoch = epoch + 1
        sampler = getattr(train_loader, "sampler", None)
        if hasattr(sampler, "set_epoch"):
            sampler.set_epoch(epoch)
        model.train()
        averages = RunningAverages()
        optimizer.zero_grad(set_to_none=True)
        epoch_start = time.perf_counter()
        epoch_examples = epoch_tokens = batches = 0
        epoch_train_s = 0.0
        last_time = time.perf_counter()
        pending = False

        def optimizer_step() -> float:
            nonlocal pending
            if hook is not None:
                norm = hook(optimizer, train_config)
            else:
                norm = _stock_optimizer_step(state, model, train_config)
            if scheduler is not None:
                scheduler.step()
            optimizer.zero_grad(set_to_none=True)
            state.global_step += 1
            pending = False
            return norm

        prefetch = getattr(model, "prefetch_batch", None)
        iterator = iter(train_loader)
        upcoming = next(iterator, _END)
        batch_idx = -1
        while upcoming is not _END:
            batch = upcoming
            batch_idx += 1
            upcoming = next(iterator, _END)
            if sync_every_batch:
                synchronize()
            timer = DeviceTimer(state.device)
            timer.start()
            wall0 = time.perf_counter()
            state.batch_step += 1
            batches += 1
            announce = getattr(model, "announce_batch", None)
            if announce is not None and upcoming is not _END:
                announce(upcoming)
            amp = torch.amp.autocast("cuda") if state.scaler is not None else nullcontext()
            with amp:
                loss, batch_metrics = batch_step(model, batch, state.device)
                scaled = loss / accum
            if state.scaler is not None:
                state.scaler.scale(scaled).backward()
            else:
                scaled.backward()
            pending = True
            did_step = (batch_idx + 1) % accum == 0
            norm = optimizer_step() if did_step else 0.0
            if prefetch is not None and upcoming is not _END:
                prefetch(upcoming)  # host planning of the next batch overlaps this step's kernels
            timer.stop()
            loss_value = float(loss.detach().float().cpu())  # the step's one host read
            if sync_every_batch:
                synchronize()
                duration = max(time.perf_counter() - wall0, 1e-9)
            else:
                duration = max(timer.seconds(), 1e-9)
            train_s += duration
            epoch_train_s += duration
            elapsed = max(time.perf_counter() - last_time, 1e-9)
            last_time = time.perf_counter()
            examples, tokens = int(batch_metrics.get("examples", 0)), int(batch_metrics.get("tokens", 0))
            epoch_examples += examples
            epoch_tokens += tokens
            sequences += examples
            processed_tokens += tokens
            metrics = {
                "train_loss": loss_value, "perplexity": perplexity(loss_value),
                "learning_rate": float(optimizer.param_groups[0]["lr"]), "grad_norm": float(norm),
                "examples_per_second": examples / elapsed, "tokens_per_second": tokens / elapsed,
                "gpu_memory_allocated": cuda_memory_allocated(state.device),
                "train_batch_duration_seconds": duration,
            }
            metrics.update(validated_extra_metrics(batch_metrics.get("metrics"), set(metrics)))
            averages.update(metrics, weight=max(examples, 1))
            state.logger.log_metrics({**metrics, "epoch": epoch + 1, "batch_in_epoch": batch_idx + 1,
                                      "optimizer_step": state.global_step, "optimizer_updated": float(did_step)},
                                     state.batch_step, "train_batch")
            if did_step:
                if state.global_step % max(train_config.log_every_steps, 1) == 0:
                    state.logger.log_metrics(metrics, state.global_step, "train")
                if eval_step and val_loader is not None and state.global_step % max(train_config.eval_every_steps, 1) == 0:
                    last_val, took = timed_evaluation(val_loader, "val")
                    val_s += took
                    last_val_step = state.global_step
                    state.logger.log_metrics(last_val, state.global_step, "val")
                    if _validation_checkpoint(state, last_val, epoch):
                        stop = True
                if state.global_step % max(train_config.save_every_steps, 1) == 0:
                    save_training_state(state, state.checkpoint.latest_path, epoch)
            if stop or (train_config.max_steps is not None and state.global_step >= train_config.max_steps):
                stop = True
                break

        if pending and not stop:
            optimizer_step()
            if train_config.max_steps is not None and state.global_step >= train_config.max_steps:
                stop = True
        epoch_metrics = averages.compute()
        took = max(time.perf_counter() - epoch_start, 1e-9)
        if "train_loss" in epoch_metrics:
            epoch_metrics["perplexity"] = perplexity(epoch_metrics["train_loss"])
        epoch_metrics.update({"examples_per_second": epoch_examples / took, "tokens_per_second": epoch_tokens / took,
                              "epoch": epoch + 1, "batches": batches, "batch_step": state.batch_step,
                              "optimizer_step": state.global_step, "examples": epoch_examples,
                              "tokens": epoch_tokens, "duration_seconds": took,
                              "train_duration_seconds": epoch_train_s})
        state.epoch_history.append(dict(epoch_metrics))
        state.logger.log_metrics(epoch_metrics, epoch + 1, "train_epoch")
        if eval_step and val_loader is not None:
            if last_val_step != state.global_step:
                last_val, took_v = timed_evaluation(val_loader, "val")
                val_s += took_v
                last_val_step = state.global_step
                state.logger.log_metrics(last_val, state.global_step, "val")
                if _validation_checkpoint(state, last_val, epoch + 1):
                    stop = True
            state.logger.log_metrics({**last_val, "epoch": epoch + 1, "optimizer_step": state.global_step,
                                      "validation_duration_seconds": last_val.get("val_duration_seconds", 0.0)},
                                     epoch + 1, "val_epoch")

    test_metrics: dict = {}
    if eval_step and test_loader is not None:
        test_metrics, test_s = timed_evaluation(test_loader, "test")
        state.logger.log_metrics(test_metrics, state.global_step, "test")
    synchronize()
    timing = {
        "wall_clock_seconds": max(time.perf_counter() - run_start, 1e-9), "train_duration_seconds": train_s,
        "validation_duration_seconds": val_s, "test_duration_seconds": test_s,
        "processed_tokens": processed_tokens, "sequences_seen": sequences, "optimizer_steps": state.global_step,
        "optimizer_steps_per_second": state.global_step / max(train_s, 1e-9),
        "training_tokens_per_second": processed_tokens / max(train_s, 1e-9),
    }
    state.logger.log_metrics(timing, state.global_step, "run")
    save_training_state(state, state.checkpoint.latest_path, last_epoch)
    close_training_state(state)
    return {"state": state, "model": model, "optimizer": optimizer, "scheduler": scheduler,
            "global_step": state.global_step, "batch_step": state.batch_step, "best_val_loss": state.best_val_loss,
            "train_metrics": epoch_metrics, "epoch_metrics": list(state.epoch_history), "val_metrics": last_val,
            "test_metrics": test_metrics, "checkpoint_dir": state.checkpoint.checkpoint_dir, "timing_metrics": timing}
