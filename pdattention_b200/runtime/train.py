"""Training engine: a loop object that keeps the device busy and reads results late.

What it does (the contract of the reference engine, ``src/common/train.py:24-486``):
AdamW with a linear-warmup ``LambdaLR``; gradient accumulation; per optimizer
step the gradient norm, clipping and the scheduler; validation and checkpoints
on an optimizer-step cadence (``latest.pt`` on every validation, on
``save_every_steps`` and at the end, ``best.pt`` when validation improves);
early stopping; end-of-epoch validation; a final test pass; run timing metrics;
the same logged splits and metric names.

How it does it differs.  A step is *issued*: batch step, backward and (when the
accumulation window closes) the optimizer update are queued on the device, and
the step's loss and gradient norm are copied into pinned host memory behind an
event.  The host reads them only after the NEXT step has been issued, so the
device always has a step queued and the host never waits for the GPU between
steps.  Anything that must observe a finished step (validation, a checkpoint,
early stopping, the end of an epoch) first drains the pending step, so logs and
checkpoints come out in the same order as with an immediate read.  A model may
provide ``optimizer_step_hook`` (the device path's fused clip + AdamW + data
parallel reduction) in place of the stock clip/step sequence, and
``announce_batch`` / ``prefetch_batch`` to plan the next batch on the host while
the current one runs.  Checkpoints and loggers are rank-0 only under
``torch.distributed``.
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


def _dist_active() -> bool:
    return torch.distributed.is_available() and torch.distributed.is_initialized()


def _rank() -> int:
    return torch.distributed.get_rank() if _dist_active() else 0


def _world() -> int:
    return torch.distributed.get_world_size() if _dist_active() else 1


@dataclass
class TrainingState:
    """Everything a run carries between steps, resumes and checkpoints."""

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
    return ("cuda" if torch.cuda.is_available() else "cpu") if device == "auto" else device


def seed_everything(seed: int) -> None:
    for seeder in (random.seed, np.random.seed, torch.manual_seed):
        seeder(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)


def move_batch(batch, device: str, non_blocking: bool = False):
    """``batch`` with every tensor (in nested dicts / lists / tuples) moved to ``device``."""
    if torch.is_tensor(batch):
        return batch.to(device, non_blocking=non_blocking)
    if isinstance(batch, (list, tuple)):
        return type(batch)(move_batch(v, device, non_blocking) for v in batch)
    if isinstance(batch, dict):
        return {k: move_batch(v, device, non_blocking) for k, v in batch.items()}
    return batch


def warmup_lambda(warmup_steps: int):
    """LambdaLR factor: linear warm-up over ``warmup_steps`` (step 0 counts as 1), then 1."""
    return lambda step: (max(step, 1) / warmup_steps) if warmup_steps and step < warmup_steps else 1.0


def _default_optimizer(model, train_config):
    build = getattr(model, "build_optimizer", None)
    if build is not None:
        optimizer = build(train_config)
        if _world() > 1 and getattr(model, "_device_runtime", None) is not None:
            from ..parallel.dp import attach_data_parallel

            # fused peer-memory gradient average, overlapped with the backward unless micro-batches
            # accumulate (a block's gradient is final only after the last micro-batch)
            attach_data_parallel(model, optimizer, _world(),
                                 overlap=False if int(train_config.grad_accum_steps) > 1 else None)
        return optimizer
    return torch.optim.AdamW(model.parameters(), lr=train_config.learning_rate, weight_decay=train_config.weight_decay)


def create_training_state(model, train_config, *, optimizer=None, scheduler=None,
                          checkpoint_extra: Callable[[], dict] | None = None) -> TrainingState:
    seed_everything(train_config.seed)
    device = resolve_device(train_config.device)
    model.to(device)
    broadcast_parameters(model)  # data parallel: every rank starts from rank 0's weights
    if getattr(model, "after_load_state", None) is not None:
        model.after_load_state()
    optimizer = optimizer if optimizer is not None else _default_optimizer(model, train_config)
    if scheduler is None:
        scheduler = torch.optim.lr_scheduler.LambdaLR(optimizer, warmup_lambda(train_config.warmup_steps))
    run_dir = Path(train_config.output_dir) / train_config.experiment_name
    logger = build_logger(train_config, run_dir, rank=_rank())
    logger.log_config(train_config)
    fp16 = train_config.mixed_precision and device.startswith("cuda") and not getattr(model, "bf16_native", False)
    state = TrainingState(model=model, train_config=train_config, device=device, optimizer=optimizer,
                          scheduler=scheduler, run_dir=run_dir, checkpoint=ModelCheckpoint(run_dir / "checkpoints"),
                          logger=logger, scaler=torch.amp.GradScaler("cuda") if fp16 else None,
                          early_stopping=EarlyStopping(train_config.early_stopping_patience),
                          checkpoint_extra=checkpoint_extra)
    if train_config.resume_from:
        resume_training_state(state, train_config.resume_from)
    return state


def resume_training_state(state: TrainingState, path) -> dict:
    payload = load_checkpoint(path, state.model, state.optimizer, state.scheduler, map_location=state.device)
    state.start_epoch = int(payload.get("epoch", 0))
    state.global_step = int(payload.get("global_step", 0))
    state.batch_step = int(payload.get("batch_step", state.global_step))
    state.best_val_loss = state.early_stopping.best = float(payload.get("best_val_loss", float("inf")))
    if getattr(state.model, "after_load_state", None) is not None:
        state.model.after_load_state()
    return payload


def save_training_state(state: TrainingState, path, epoch: int) -> Path:
    """Write the checkpoint payload (rank 0 only; other ranks return the path unwritten)."""
    path = Path(path)
    if _rank() != 0:
        return path
    payload = {"model": state.model.state_dict(), "optimizer": state.optimizer.state_dict(),
               "scheduler": None if state.scheduler is None else state.scheduler.state_dict(),
               "config": serializable_config(state.train_config), "epoch": epoch,
               "global_step": state.global_step, "batch_step": state.batch_step, "best_val_loss": state.best_val_loss}
    payload.update(state.checkpoint_extra() if state.checkpoint_extra else {})
    return atomic_save(payload, path)


def close_training_state(state: TrainingState) -> None:
    if not state.logger_closed:
        state.logger_closed = True
        state.logger.close()


def default_batch_step(model, batch: dict, device: str, *, ignore_index: int = -100):
    """Causal-LM step for models returning logits (or an object with ``.logits``)."""
    batch = move_batch(batch, device)
    out = model(batch["input_ids"])
    logits = out.logits if hasattr(out, "logits") else out
    loss = F.cross_entropy(logits.flatten(0, -2), batch["labels"].flatten(), ignore_index=ignore_index)
    mask = batch.get("attention_mask")
    counted = mask.sum() if mask is not None else (batch["labels"] != ignore_index).sum()
    return loss, {"tokens": int(counted.item()), "examples": int(batch["input_ids"].shape[0])}


def validated_extra_metrics(values: dict | None, reserved: set[str]) -> dict[str, float]:
    """The batch step's own scalar metrics (tensors of one element included), minus engine names."""
    out = {}
    for key, value in (values or {}).items():
        if not isinstance(key, str) or key in reserved:
            continue
        if torch.is_tensor(value):
            if value.numel() != 1:
                continue
            value = value.detach().item()
        if isinstance(value, (int, float, bool)):
            out[key] = float(value)
    return out


def average_gradients(model) -> None:
    """Data parallel: every rank's gradients become the mean over ranks (one flat all-reduce;
    gloo on CPU, NCCL on GPU).  No-op outside a process group."""
    world = _world()
    grads = [p.grad for p in model.parameters() if p.grad is not None] if world > 1 else []
    if not grads:
        return
    flat = torch.cat([g.reshape(-1).float() for g in grads])
    torch.distributed.all_reduce(flat, op=torch.distributed.ReduceOp.SUM)
    flat /= world
    for g, part in zip(grads, flat.split([g.numel() for g in grads])):
        g.copy_(part.view_as(g))


def broadcast_parameters(model, src: int = 0) -> None:
    """Start every data-parallel rank from rank ``src``'s parameters."""
    if _world() <= 1:
        return
    with torch.no_grad():
        for p in model.parameters():
            torch.distributed.broadcast(p.data, src=src)


@dataclass
class _Issued:
    """A step queued on the device whose scalars have not been read yet."""

    epoch: int
    batch_in_epoch: int
    batch_step: int
    global_step: int
    updated: bool
    learning_rate: float
    loss: torch.Tensor
    norm: object
    batch_metrics: dict
    timer: DeviceTimer
    wall_start: float
    issued_at: float
    host: torch.Tensor | None = None
    ready: object = None

    def stage(self, cuda: bool) -> None:
        """Start the asynchronous copy of the loss and gradient norm to pinned host memory."""
        norm = self.norm if torch.is_tensor(self.norm) else torch.tensor(float(self.norm), device=self.loss.device)
        pair = torch.stack([self.loss.detach().float().reshape(()), norm.detach().float().reshape(())])
        if cuda and pair.is_cuda:
            self.host = torch.empty(2, dtype=torch.float32, pin_memory=True)
            self.host.copy_(pair, non_blocking=True)
            self.ready = torch.cuda.Event()
            self.ready.record()
        else:
            self.host = pair

    def read(self) -> tuple[float, float]:
        if self.ready is not None:
            self.ready.synchronize()
        return float(self.host[0]), float(self.host[1])


class _TrainingLoop:
    def __init__(self, state: TrainingState, *, train_loader, val_loader, test_loader, batch_step, eval_step,
                 sync_every_batch: bool | None):
        self.state, self.cfg = state, state.train_config
        self.model, self.optimizer, self.scheduler = state.model, state.optimizer, state.scheduler
        self.train_loader, self.val_loader, self.test_loader = train_loader, val_loader, test_loader
        self.batch_step, self.eval_step = batch_step, eval_step
        self.hook = getattr(self.model, "optimizer_step_hook", None)
        self.sync_every_batch = self.hook is None if sync_every_batch is None else sync_every_batch
        self.cuda = state.device.startswith("cuda") and torch.cuda.is_available()
        self.accum = max(int(self.cfg.grad_accum_steps), 1)
        self.stop = bool(self.cfg.max_steps is not None and state.global_step >= self.cfg.max_steps)
        self.pending: _Issued | None = None
        self.last_val: dict = {}
        self.last_val_step = -1
        self.epoch_metrics: dict = {}
        self.seconds = {"train": 0.0, "val": 0.0, "test": 0.0}
        self.tokens = self.sequences = 0
        self.last_epoch = state.start_epoch

    # -- helpers -------------------------------------------------------------------
    def _sync(self) -> None:
        if self.cuda:
            torch.cuda.synchronize()

    def _evaluate(self, loader, split: str) -> dict:
        self._sync()
        t0 = time.perf_counter()
        values = self.eval_step(self.model, loader, self.state.device, split=split)
        self._sync()
        values[f"{split}_duration_seconds"] = max(time.perf_counter() - t0, 1e-9)
        self.seconds["val" if split == "val" else split] += values[f"{split}_duration_seconds"]
        return values

    def _update(self):
        """Clip + update (+ scheduler), zero the gradients; returns the norm (maybe on the device)."""
        if self.hook is not None:
            norm = self.hook(self.optimizer, self.cfg)
        else:
            average_gradients(self.model)
            if self.state.scaler is not None:
                self.state.scaler.unscale_(self.optimizer)
            norm = grad_norm(self.model.parameters())
            if self.cfg.max_grad_norm:
                torch.nn.utils.clip_grad_norm_(self.model.parameters(), self.cfg.max_grad_norm)
            if self.state.scaler is not None:
                self.state.scaler.step(self.optimizer)
                self.state.scaler.update()
            else:
                self.optimizer.step()
        if self.scheduler is not None:
            self.scheduler.step()
        self.optimizer.zero_grad(set_to_none=True)
        self.state.global_step += 1
        return norm

    def _validate_and_checkpoint(self, epoch_for_checkpoint: int) -> None:
        state = self.state
        self.last_val = self._evaluate(self.val_loader, "val")
        self.last_val_step = state.global_step
        state.logger.log_metrics(self.last_val, state.global_step, "val")
        val_loss = self.last_val.get("val_loss", self.last_val.get("loss", float("inf")))
        improved = val_loss < state.best_val_loss
        if improved:
            state.best_val_loss = val_loss
        save_training_state(state, state.checkpoint.latest_path, epoch_for_checkpoint)
        if improved:
            save_training_state(state, state.checkpoint.best_path, epoch_for_checkpoint)
        if state.early_stopping.update(val_loss):
            self.stop = True

    # -- one step --------------------------------------------------------------------
    def _issue(self, epoch: int, index: int, batch, upcoming) -> _Issued:
        state, model = self.state, self.model
        if self.sync_every_batch:
            self._sync()
        timer = DeviceTimer(state.device)
        timer.start()
        wall_start = time.perf_counter()
        state.batch_step += 1
        if upcoming is not None and getattr(model, "announce_batch", None) is not None:
            model.announce_batch(upcoming)
        with torch.amp.autocast("cuda") if state.scaler is not None else nullcontext():
            loss, batch_metrics = self.batch_step(model, batch, state.device)
            scaled = loss / self.accum
        (state.scaler.scale(scaled) if state.scaler is not None else scaled).backward()
        self._unapplied = True
        updated = (index + 1) % self.accum == 0
        norm = self._update() if updated else 0.0
        if updated:
            self._unapplied = False
        if upcoming is not None and getattr(model, "prefetch_batch", None) is not None:
            model.prefetch_batch(upcoming)  # host planning of the next batch overlaps this step's kernels
        timer.stop()
        step = _Issued(epoch, index, state.batch_step, state.global_step, updated,
                       float(self.optimizer.param_groups[0]["lr"]), loss, norm, batch_metrics, timer, wall_start,
                       time.perf_counter())
        step.stage(self.cuda)
        return step

    def _record(self, step: _Issued, averages: RunningAverages, counters: dict) -> None:
        """Read a finished step's scalars and log them (train_batch, and train on the log cadence)."""
        state = self.state
        loss, norm = step.read()
        if self.sync_every_batch:
            self._sync()
            duration = max(time.perf_counter() - step.wall_start, 1e-9)
        else:
            duration = max(step.timer.seconds(), 1e-9)
        elapsed = max(step.issued_at - counters["last_issue_end"], 1e-9)
        counters["last_issue_end"] = step.issued_at
        examples, tokens = int(step.batch_metrics.get("examples", 0)), int(step.batch_metrics.get("tokens", 0))
        self.seconds["train"] += duration
        counters["train_s"] += duration
        counters["examples"] += examples
        counters["tokens"] += tokens
        self.sequences += examples
        self.tokens += tokens
        metrics = {"train_loss": loss, "perplexity": perplexity(loss), "learning_rate": step.learning_rate,
                   "grad_norm": norm, "examples_per_second": examples / elapsed, "tokens_per_second": tokens / elapsed,
                   "gpu_memory_allocated": cuda_memory_allocated(state.device),
                   "train_batch_duration_seconds": duration}
        metrics.update(validated_extra_metrics(step.batch_metrics.get("metrics"), set(metrics)))
        averages.update(metrics, weight=max(examples, 1))
        state.logger.log_metrics({**metrics, "epoch": step.epoch + 1, "batch_in_epoch": step.batch_in_epoch + 1,
                                  "optimizer_step": step.global_step, "optimizer_updated": float(step.updated)},
                                 step.batch_step, "train_batch")
        if step.updated and step.global_step % max(self.cfg.log_every_steps, 1) == 0:
            state.logger.log_metrics(metrics, step.global_step, "train")

    def _drain(self, averages, counters) -> None:
        if self.pending is not None:
            step, self.pending = self.pending, None
            self._record(step, averages, counters)

    def _after_update(self, epoch: int) -> None:
        """Validation / checkpoint cadence of the optimizer step that just completed."""
        step = self.state.global_step
        if self.eval_step and self.val_loader is not None and step % max(self.cfg.eval_every_steps, 1) == 0:
            self._validate_and_checkpoint(epoch)
        if step % max(self.cfg.save_every_steps, 1) == 0:
            save_training_state(self.state, self.state.checkpoint.latest_path, epoch)

    def _needs_observation(self, step: _Issued) -> bool:
        """Whether anything right after this step must see its finished values first."""
        if self.sync_every_batch or not step.updated:
            return self.sync_every_batch
        g = step.global_step
        return (bool(self.eval_step and self.val_loader is not None and g % max(self.cfg.eval_every_steps, 1) == 0)
                or g % max(self.cfg.save_every_steps, 1) == 0
                or (self.cfg.max_steps is not None and g >= self.cfg.max_steps))

    # -- epochs ------------------------------------------------------------------------
    def _epoch(self, epoch: int) -> None:
        state, model = self.state, self.model
        sampler = getattr(self.train_loader, "sampler", None)
        if hasattr(sampler, "set_epoch"):
            sampler.set_epoch(epoch)
        model.train()
        averages = RunningAverages()
        self.optimizer.zero_grad(set_to_none=True)
        started = time.perf_counter()
        counters = {"last_issue_end": started, "train_s": 0.0, "examples": 0, "tokens": 0}
        self._unapplied = False
        batches = 0
        iterator = iter(self.train_loader)
        marker = object()
        upcoming = next(iterator, marker)
        index = -1
        while upcoming is not marker:
            batch, upcoming = upcoming, next(iterator, marker)
            index += 1
            batches += 1
            step = self._issue(epoch, index, batch, None if upcoming is marker else upcoming)
            self._drain(averages, counters)  # the previous step, read after this one was queued
            self.pending = step
            if self._needs_observation(step):
                self._drain(averages, counters)
            if step.updated:
                self._after_update(epoch)
            if self.stop or (self.cfg.max_steps is not None and state.global_step >= self.cfg.max_steps):
                self.stop = True
                break
        self._drain(averages, counters)
        if self._unapplied and not self.stop:  # a partial accumulation window at the end of the epoch
            self._update()
            if self.cfg.max_steps is not None and state.global_step >= self.cfg.max_steps:
                self.stop = True
        self._close_epoch(epoch, averages, counters, batches, started)

    def _close_epoch(self, epoch, averages, counters, batches, started) -> None:
        state = self.state
        took = max(time.perf_counter() - started, 1e-9)
        metrics = averages.compute()
        if "train_loss" in metrics:
            metrics["perplexity"] = perplexity(metrics["train_loss"])
        metrics.update({"examples_per_second": counters["examples"] / took,
                        "tokens_per_second": counters["tokens"] / took, "epoch": epoch + 1, "batches": batches,
                        "batch_step": state.batch_step, "optimizer_step": state.global_step,
                        "examples": counters["examples"], "tokens": counters["tokens"], "duration_seconds": took,
                        "train_duration_seconds": counters["train_s"]})
        self.epoch_metrics = metrics
        state.epoch_history.append(dict(metrics))
        state.logger.log_metrics(metrics, epoch + 1, "train_epoch")
        if self.eval_step and self.val_loader is not None:
            if self.last_val_step != state.global_step:
                self._validate_and_checkpoint(epoch + 1)
            state.logger.log_metrics({**self.last_val, "epoch": epoch + 1, "optimizer_step": state.global_step,
                                      "validation_duration_seconds": self.last_val.get("val_duration_seconds", 0.0)},
                                     epoch + 1, "val_epoch")

    def run(self, run_start: float) -> dict:
        state = self.state
        for epoch in range(state.start_epoch, self.cfg.epochs):
            if self.stop:
                break
            self.last_epoch = epoch + 1
            self._epoch(epoch)
        test_metrics: dict = {}
        if self.eval_step and self.test_loader is not None:
            test_metrics = self._evaluate(self.test_loader, "test")
            state.logger.log_metrics(test_metrics, state.global_step, "test")
        self._sync()
        train_s = self.seconds["train"]
        timing = {"wall_clock_seconds": max(time.perf_counter() - run_start, 1e-9), "train_duration_seconds": train_s,
                  "validation_duration_seconds": self.seconds["val"], "test_duration_seconds": self.seconds["test"],
                  "processed_tokens": self.tokens, "sequences_seen": self.sequences,
                  "optimizer_steps": state.global_step,
                  "optimizer_steps_per_second": state.global_step / max(train_s, 1e-9),
                  "training_tokens_per_second": self.tokens / max(train_s, 1e-9)}
        state.logger.log_metrics(timing, state.global_step, "run")
        save_training_state(state, state.checkpoint.latest_path, self.last_epoch)
        close_training_state(state)
        return {"state": state, "model": self.model, "optimizer": self.optimizer, "scheduler": self.scheduler,
                "global_step": state.global_step, "batch_step": state.batch_step, "best_val_loss": state.best_val_loss,
                "train_metrics": self.epoch_metrics, "epoch_metrics": list(state.epoch_history),
                "val_metrics": self.last_val, "test_metrics": test_metrics,
                "checkpoint_dir": state.checkpoint.checkpoint_dir, "timing_metrics": timing}


def train_model(*, model, train_config, train_loader, val_loader=None, test_loader=None, optimizer=None,
                scheduler=None, batch_step=default_batch_step, eval_step=None, checkpoint_extra=None,
                state: TrainingState | None = None, sync_every_batch: bool | None = None):
    """Epochs of ``batch_step`` + backward + optimizer updates with evaluation / checkpoint cadence.

    ``sync_every_batch`` (default: only for models without a fused optimizer hook)
    brackets every batch with a device synchronise and times it on the host
    clock, as the reference engine does; otherwise batches are timed with CUDA
    events and their losses read one step late.
    """
    run_start = time.perf_counter()
    state = state or create_training_state(model, train_config, optimizer=optimizer, scheduler=scheduler,
                                           checkpoint_extra=checkpoint_extra)
    if checkpoint_extra is not None:
        state.checkpoint_extra = checkpoint_extra
    loop = _TrainingLoop(state, train_loader=train_loader, val_loader=val_loader, test_loader=test_loader,
                         batch_step=batch_step, eval_step=eval_step, sync_every_batch=sync_every_batch)
    return loop.run(run_start)
