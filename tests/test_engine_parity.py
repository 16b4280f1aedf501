"""The training engine against the reference engine (``src/common/train.py``) on CPU.

Same tiny language model, data, seeds and settings (gradient accumulation with a
partial final window, validation and checkpoint cadence, early stopping off, a
step cap): the sequence of logged records (split, step, metric names), the
checkpoint counters and the trained weights must match.
"""

import json

import pytest
import torch

from pdattention_b200.config import BaseTrainConfig
from pdattention_b200.runtime.checkpointing import read_checkpoint
from pdattention_b200.runtime.train import train_model


class _LM(torch.nn.Module):
    def __init__(self, vocab=37, d=16):
        super().__init__()
        self.emb = torch.nn.Embedding(vocab, d)
        self.out = torch.nn.Linear(d, vocab)

    def forward(self, ids):
        return self.out(torch.tanh(self.emb(ids)))


def _loader(seed, n=11, t=9):
    gen = torch.Generator().manual_seed(seed)
    ids = torch.randint(1, 37, (n, t), generator=gen)
    rows = [{"input_ids": ids[i], "labels": torch.roll(ids[i], -1), "attention_mask": torch.ones(t, dtype=torch.long)}
            for i in range(n)]
    return torch.utils.data.DataLoader(rows, batch_size=3, shuffle=False)


def _eval(model, loader, device, split="val"):
    model.eval()
    with torch.no_grad():
        losses = [torch.nn.functional.cross_entropy(model(b["input_ids"]).flatten(0, 1), b["labels"].flatten()).item()
                  for b in loader]
    model.train()
    return {f"{split}_loss": sum(losses) / len(losses)}


def _settings(out):
    return dict(output_dir=str(out), experiment_name="x", epochs=3, max_steps=5, grad_accum_steps=2,
                eval_every_steps=2, save_every_steps=3, log_every_steps=1, use_tensorboard=False,
                save_metric_plots=False, learning_rate=3e-2, warmup_steps=2, device="cpu", seed=5)


def _records(path):
    data = json.loads(path.read_text())["records"]
    return [(r["split"], r["step"], sorted(r["metrics"]), {k: r.get(k) for k in ("epoch", "batch_in_epoch", "optimizer_step")})
            for r in data]


def test_engine_matches_reference_engine(ref, tmp_path):
    import importlib

    ref_train = importlib.import_module("common.train")
    ref_config = importlib.import_module("common.config")
    torch.manual_seed(0)
    ours_model = _LM()
    theirs_model = _LM()
    theirs_model.load_state_dict(ours_model.state_dict())
    ours = train_model(model=ours_model, train_config=BaseTrainConfig(**_settings(tmp_path / "ours")),
                       train_loader=_loader(1), val_loader=_loader(2, n=4), test_loader=_loader(3, n=4),
                       eval_step=_eval)
    theirs = ref_train.train_model(model=theirs_model, train_config=ref_config.TrainConfig(**_settings(tmp_path / "ref")),
                                   train_loader=_loader(1), val_loader=_loader(2, n=4), test_loader=_loader(3, n=4),
                                   eval_step=_eval)
    assert ours["global_step"] == theirs["global_step"] and ours["batch_step"] == theirs["batch_step"]
    assert ours["best_val_loss"] == pytest.approx(theirs["best_val_loss"], rel=1e-6)
    mine, reference = _records(tmp_path / "ours" / "x" / "metrics.json"), _records(tmp_path / "ref" / "x" / "metrics.json")
    drop = {"wall_clock_seconds"}  # keys present in both; compare names only
    assert [(s, st, [k for k in ks if k not in drop], d) for s, st, ks, d in mine] == \
           [(s, st, [k for k in ks if k not in drop], d) for s, st, ks, d in reference]
    for a, b in zip(ours_model.parameters(), theirs_model.parameters()):
        assert torch.allclose(a, b, atol=1e-6), (a - b).abs().max()
    for name in ("latest.pt", "best.pt"):
        p, q = read_checkpoint(tmp_path / "ours" / "x" / "checkpoints" / name), \
            read_checkpoint(tmp_path / "ref" / "x" / "checkpoints" / name)
        assert {k: p[k] for k in ("epoch", "global_step", "batch_step")} == \
               {k: q[k] for k in ("epoch", "global_step", "batch_step")}
