"""Autograd functions over the sm_100a kernels (bf16 activations, fp32 accumulation).

Weights enter these functions as ``WeightSlot`` objects: the bf16 compute copy
``w`` (refreshed by the fused AdamW step) and ``gw`` / ``gb``, views into the
flat bf16 gradient buffer that the optimizer (and the data-parallel reduction)
reads.  Weight-gradient GEMMs write straight into those views (``beta = 1``
when accumulating micro-batches), so there is no per-parameter gradient
allocation or copy.  Every function requires CUDA tensors and the built
extension; the CPU path of the framework is the object path in ``models``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from ._ext import require


@dataclass
class WeightSlot:
    """Compute copy and gradient views of one linear / norm / embedding parameter set."""

    w: torch.Tensor
    b: torch.Tensor | None = None
    gw: torch.Tensor | None = None
    gb: torch.Tensor | None = None
    fresh: list = field(default_factory=lambda: [True])  # next gradient write overwrites (beta = 0)

    def grad_beta(self) -> float:
        beta = 0.0 if self.fresh[0] else 1.0
        self.fresh[0] = False
        return beta


@dataclass(frozen=True)
class DropoutSpec:
    """One dropout site of one call: probability ``p`` and the Philox stream ``(seed, offset)``
    the kernels draw the mask from (forward and backward regenerate the same mask)."""

    p: float
    seed: int
    offset: int


class DropoutStreams:
    """Hands out a fresh ``DropoutSpec`` per dropout site and call (the offset counts calls)."""

    def __init__(self, seed: int | None = None):
        self.seed = int(torch.randint(0, 2 ** 62, (1,)).item()) if seed is None else int(seed)
        self.offset = 0

    def next(self, p: float) -> DropoutSpec | None:
        if p <= 0.0:
            return None
        self.offset += 1
        return DropoutSpec(float(p), self.seed, self.offset)


def _drop(x: torch.Tensor, spec: DropoutSpec | None) -> torch.Tensor:
    """``x`` with the spec's mask applied (new tensor; ``x`` itself when no spec)."""
    if spec is None:
        return x
    out = torch.empty_like(x)
    require().dropout(x.contiguous(), out, spec.p, spec.seed, spec.offset)
    return out


class _DropoutAdd(torch.autograd.Function):
    """y = residual + dropout(x)."""

    @staticmethod
    def forward(ctx, residual, x, spec: DropoutSpec):
        y = torch.empty_like(x)
        require().dropout_add(residual.contiguous(), x.contiguous(), y, spec.p, spec.seed, spec.offset)
        ctx.spec = spec
        return y

    @staticmethod
    def backward(ctx, dy):
        dy = dy.contiguous()
        return dy, _drop(dy, ctx.spec), None


def dropout_add(residual: torch.Tensor, x: torch.Tensor, spec: DropoutSpec | None) -> torch.Tensor:
    if spec is None:
        return residual + x
    return _DropoutAdd.apply(residual, x, spec)


def _write_bias_grad(slot: WeightSlot, g: torch.Tensor, beta: float) -> None:
    if slot.gb is None:
        return
    summed = require().colsum(g)
    if beta == 0.0:
        slot.gb.copy_(summed)
    else:
        slot.gb.add_(summed)


def _wgrad(slot: WeightSlot, dy: torch.Tensor, x: torch.Tensor, alpha_ptr=None) -> None:
    """gw (+)= dy^T x and gb (+)= colsum(dy)."""
    if slot.gw is None:
        return
    beta = slot.grad_beta()
    ext = require()
    ext.gemm("wgrad", dy, x, slot.gw if beta else None, slot.gw, None, None, 1.0, beta, alpha_ptr)
    _write_bias_grad(slot, dy, beta)


class _Linear(torch.autograd.Function):
    """y = x W^T + b (+ residual)."""

    @staticmethod
    def forward(ctx, x, slot: WeightSlot, residual):
        ext = require()
        y = torch.empty((x.shape[0], slot.w.shape[0]), device=x.device, dtype=torch.bfloat16)
        ext.gemm("tn", x, slot.w, residual, y, slot.b, None, 1.0, 1.0 if residual is not None else 0.0, None)
        ctx.slot = slot
        ctx.has_residual = residual is not None
        ctx.save_for_backward(x)
        return y

    @staticmethod
    def backward(ctx, dy):
        (x,) = ctx.saved_tensors
        dy = dy.contiguous()
        ext = require()
        dx = torch.empty_like(x)
        ext.gemm("nn", dy, ctx.slot.w, None, dx, None, None, 1.0, 0.0, None)
        _wgrad(ctx.slot, dy, x)
        return dx, None, (dy if ctx.has_residual else None)


def linear(x: torch.Tensor, slot: WeightSlot, residual: torch.Tensor | None = None) -> torch.Tensor:
    return _Linear.apply(x, slot, residual)


class _Mlp(torch.autograd.Function):
    """y = residual + drop_out(drop_in(gelu(h W1^T + b1)) W2^T + b2) with the GELU derivative
    fused into the dgrad GEMM.  ``drop_in`` / ``drop_out`` (optional ``DropoutSpec``) are the
    vanilla blocks' dropout after the activation and on the branch output; the masks are
    regenerated in the backward (a mask commutes with the elementwise GELU derivative)."""

    @staticmethod
    def forward(ctx, h, residual, up: WeightSlot, down: WeightSlot, drop_in, drop_out):
        ext = require()
        m = h.shape[0]
        z = torch.empty((m, up.w.shape[0]), device=h.device, dtype=torch.bfloat16)
        u = torch.empty_like(z)
        ext.gemm("tn_gelu", h, up.w, None, u, up.b, z, 1.0, 0.0, None)
        if drop_in is not None:
            ext.dropout(u, u, drop_in.p, drop_in.seed, drop_in.offset)
        y = torch.empty((m, down.w.shape[0]), device=h.device, dtype=torch.bfloat16)
        if drop_out is None:
            ext.gemm("tn", u, down.w, residual, y, down.b, None, 1.0, 1.0 if residual is not None else 0.0, None)
        else:
            ext.gemm("tn", u, down.w, None, y, down.b, None, 1.0, 0.0, None)
            if residual is not None:
                ext.dropout_add(residual.contiguous(), y, y, drop_out.p, drop_out.seed, drop_out.offset)
            else:
                ext.dropout(y, y, drop_out.p, drop_out.seed, drop_out.offset)
        ctx.up, ctx.down = up, down
        ctx.drops = (drop_in, drop_out)
        ctx.has_residual = residual is not None
        ctx.save_for_backward(h, z, u)
        return y

    @staticmethod
    def backward(ctx, dy):
        h, z, u = ctx.saved_tensors
        drop_in, drop_out = ctx.drops
        dy = dy.contiguous()
        dbranch = _drop(dy, drop_out)
        ext = require()
        dz = torch.empty_like(z)
        ext.gemm("nn_dgelu", dbranch, ctx.down.w, None, dz, None, z, 1.0, 0.0, None)
        if drop_in is not None:
            ext.dropout(dz, dz, drop_in.p, drop_in.seed, drop_in.offset)
        _wgrad(ctx.down, dbranch, u)
        dh = torch.empty_like(h)
        ext.gemm("nn", dz, ctx.up.w, None, dh, None, None, 1.0, 0.0, None)
        _wgrad(ctx.up, dz, h)
        return dh, (dy if ctx.has_residual else None), None, None, None, None


def mlp(h, residual, up: WeightSlot, down: WeightSlot, drop_in: DropoutSpec | None = None,
        drop_out: DropoutSpec | None = None):
    return _Mlp.apply(h, residual, up, down, drop_in, drop_out)


class _Norm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, slot: WeightSlot, eps: float, rms: bool):
        y, mean, rstd = require().norm_fwd(x, slot.w, slot.b, eps, rms)
        ctx.slot, ctx.rms = slot, rms
        ctx.save_for_backward(x, mean, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, mean, rstd = ctx.saved_tensors
        dx, dw, db = require().norm_bwd(dy.contiguous(), x, ctx.slot.w, mean, rstd, None, ctx.rms)
        slot = ctx.slot
        if slot.gw is not None:
            beta = slot.grad_beta()
            if beta == 0.0:
                slot.gw.copy_(dw)
                if slot.gb is not None:
                    slot.gb.copy_(db)
            else:
                slot.gw.add_(dw)
                if slot.gb is not None:
                    slot.gb.add_(db)
        return dx, None, None, None


def layer_norm(x, slot: WeightSlot, eps: float = 1e-5):
    return _Norm.apply(x, slot, eps, False)


def rms_norm(x, slot: WeightSlot, eps: float = 1e-6):
    return _Norm.apply(x, slot, eps, True)


@dataclass
class MemoryView:
    """The memory keys of one attention call: pools plus per-row pool-row lists."""

    k: torch.Tensor        # [rows, width] bf16 (may be a strided view into a QKV buffer)
    v: torch.Tensor
    idx: torch.Tensor      # [B, max] int32
    length: torch.Tensor   # [B] int32


class _Attention(torch.autograd.Function):
    """One softmax over [memory (visible) ; local (causal, padding-masked)] keys."""

    @staticmethod
    def forward(ctx, qkv, heads: int, head_dim: int, memory: MemoryView | None, key_valid, scale: float,
                drop: DropoutSpec | None = None):
        b, t, width = qkv.shape
        d = heads * head_dim
        q, k, v = qkv[..., :d], qkv[..., d:2 * d], qkv[..., 2 * d:3 * d]
        mk = mv = mi = ml = None
        if memory is not None:
            mk, mv, mi, ml = memory.k, memory.v, memory.idx, memory.length
        dp, ds, do = (drop.p, drop.seed, drop.offset) if drop is not None else (0.0, 0, 0)
        out, lse = require().attention_fwd(q, k, v, heads, heads, head_dim, mk, mv, mi, ml, key_valid, scale, dp, ds,
                                           do)
        ctx.meta = (heads, head_dim, memory, scale, drop)
        ctx.save_for_backward(qkv, out, lse, key_valid if key_valid is not None else torch.empty(0))
        return out

    @staticmethod
    def backward(ctx, dout):
        qkv, out, lse, key_valid = ctx.saved_tensors
        heads, head_dim, memory, scale, drop = ctx.meta
        d = heads * head_dim
        q, k, v = qkv[..., :d], qkv[..., d:2 * d], qkv[..., 2 * d:3 * d]
        mk = mv = mi = ml = None
        if memory is not None:
            mk, mv, mi, ml = memory.k, memory.v, memory.idx, memory.length
        dp, ds, do = (drop.p, drop.seed, drop.offset) if drop is not None else (0.0, 0, 0)
        (dqkv,) = require().attention_bwd(dout.contiguous(), q, k, v, out, lse, heads, head_dim, mk, mv, mi, ml,
                                          key_valid if key_valid.numel() else None, scale, dp, ds, do)
        return dqkv, None, None, None, None, None, None


def attention(qkv: torch.Tensor, heads: int, head_dim: int, memory: MemoryView | None = None,
              key_valid: torch.Tensor | None = None, scale: float | None = None,
              drop: DropoutSpec | None = None) -> torch.Tensor:
    """``qkv`` ``[B, T, 3*H*Dh]`` (q, k, v packed per token) -> ``[B, T, H*Dh]``; ``drop`` applies
    dropout to the attention probabilities (local attention only)."""
    scale = 1.0 / math.sqrt(head_dim) if scale is None else scale
    return _Attention.apply(qkv, heads, head_dim, memory, key_valid, scale, drop)


class _LmHeadLoss(torch.autograd.Function):
    """Mean cross-entropy of ``hidden @ W^T`` over labels != ignore_index (logits never leave the kernel pair)."""

    @staticmethod
    def forward(ctx, hidden, slot: WeightSlot, labels, vocab: int, ignore_index: int):
        ext = require()
        logits = torch.empty((hidden.shape[0], slot.w.shape[0]), device=hidden.device, dtype=torch.bfloat16)
        ext.gemm("tn", hidden, slot.w, None, logits, None, None, 1.0, 0.0, None)
        row_loss, row_valid = ext.cross_entropy(logits, labels, vocab, ignore_index)
        count = row_valid.sum()
        loss = row_loss.sum() / count.clamp_min(1.0)
        ctx.slot = slot
        ctx.save_for_backward(hidden, logits, count)
        return loss

    @staticmethod
    def backward(ctx, dloss):
        hidden, glogits, count = ctx.saved_tensors
        scale = (dloss.float() / count.clamp_min(1.0)).reshape(1).contiguous()
        ext = require()
        dh = torch.empty_like(hidden)
        ext.gemm("nn", glogits, ctx.slot.w, None, dh, None, None, 1.0, 0.0, scale)
        if ctx.slot.gw is not None:
            beta = ctx.slot.grad_beta()
            ext.gemm("wgrad", glogits, hidden, ctx.slot.gw if beta else None, ctx.slot.gw, None, None, 1.0, beta,
                     scale)
        return dh, None, None, None, None


def lm_head_loss(hidden, slot: WeightSlot, labels, vocab: int, ignore_index: int = 0):
    return _LmHeadLoss.apply(hidden, slot, labels, vocab, ignore_index)


def lm_head_logits(hidden, slot: WeightSlot) -> torch.Tensor:
    out = torch.empty((hidden.shape[0], slot.w.shape[0]), device=hidden.device, dtype=torch.bfloat16)
    require().gemm("tn", hidden, slot.w, None, out, None, None, 1.0, 0.0, None)
    return out
