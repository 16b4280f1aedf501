"""Device execution path for TinyGPT-PRA (filled in by the sm_100a kernel layer)."""

from __future__ import annotations

import torch

from .tiny import TinyPRAModel


def prepare_model(cfg, device) -> TinyPRAModel:
    """Build a model on ``device``; on CUDA it is wrapped for the bf16 device path."""
    model = TinyPRAModel(cfg)
    return model.to(device)


def device_batch_step(*args, **kwargs):
    raise NotImplementedError


def pra_attention_device(layer, x, attention_mask):
    raise NotImplementedError
