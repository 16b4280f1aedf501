"""Standalone training / evaluation entry points around ``PRAStandaloneTrainer``.

Same command surface as the reference's ``scripts/train_standalone.py`` and
``scripts/eval_standalone.py``::

    python -m pdattention_b200.standalone train --config config/config.yml --model standalone_tiny
    python -m pdattention_b200.standalone eval --checkpoint out/<run>/best.pt [--predictions-jsonl ...]

The YAML's ``standalone`` (or top-level) section fills ``TrainConfig``; its ``model`` /
``pra`` sections fill ``PRAConfig`` (the vocabulary comes from the data module's tokenizer).
"""

from __future__ import annotations

import argparse
from dataclasses import fields
from pathlib import Path

from .cli import load_config
from .config import CacheServiceConfig, PRAConfig, ResolverServiceConfig, TrainConfig
from .data import PRADataModule
from .trainer import PRAStandaloneTrainer

def train_config_from_dict(raw: dict) -> TrainConfig:
    section = raw.get("standalone", raw)
    names = {f.name for f in fields(TrainConfig)}
    values = {k: v for k, v in section.items() if k in names}
    values["resolver_config"] = ResolverServiceConfig.from_value(values.get("resolver_config", raw.get("resolver")))
    values["cache_config"] = CacheServiceConfig.from_value(values.get("cache_config", raw.get("cache")))
    return TrainConfig(**values)


def model_config_from_dict(raw: dict, vocab_size: int, train_cfg: TrainConfig) -> PRAConfig:
    """PRAConfig from the YAML's ``pra`` (or ``model``) section plus the standalone model shape."""
    model = raw.get("model", {})
    pra = raw.get("pra", model)
    values = {f.name: pra[f.name] for f in fields(PRAConfig) if f.name in pra}
    values.update(
        vocab_size=vocab_size,
        d_model=int(model.get("d_model", 128)),
        n_heads=int(model.get("n_heads", 4)),
        n_layers=int(model.get("n_layers", 4)),
        n_vanilla_layers=int(model.get("n_vanilla_layers", 0)),
        n_mixed_layers=int(model.get("n_mixed_layers", 0)),
        d_ff=int(model["d_ff"]) if model.get("d_ff") is not None else None,
        max_seq_len=train_cfg.max_seq_len,
        dropout=float(model.get("dropout", 0.0)),
        model_variant=str(model.get("model_variant", "custom")),
        pra_layer_ids=tuple(pra.get("pra_layer_ids", (2, 3))),
        trigger_threshold=float(pra.get("trigger_threshold", 0.2)),
        memory_transport=str(pra.get("memory_transport", "native_kv")),
        memory_alpha=float(pra.get("memory_alpha", 0.5)),
        batch_size=train_cfg.batch_size,
        lr=train_cfg.learning_rate,
        steps=train_cfg.epochs,
        device=train_cfg.device,
    )
    return PRAConfig(**values)


def build_trainer(config_path: str, output_dir: str | None = None, resume_from: str | None = None,
                  device: str | None = None, model_name: str = "standalone_tiny") -> PRAStandaloneTrainer:
    raw = load_config(config_path, model_name=model_name)
    train_cfg = train_config_from_dict(raw)
    if output_dir:
        train_cfg.output_dir = output_dir
    if resume_from:
        train_cfg.resume_from = resume_from
    if device:
        train_cfg.device = device
    dm = PRADataModule(dataset_stage=train_cfg.dataset_stage, data_dir=train_cfg.data_dir,
                       max_examples=train_cfg.max_examples, batch_size=train_cfg.batch_size,
                       max_seq_len=train_cfg.max_seq_len, shuffle=train_cfg.shuffle, num_workers=train_cfg.num_workers,
                       pin_memory=train_cfg.pin_memory, persistent_workers=train_cfg.persistent_workers).load()
    return PRAStandaloneTrainer(model_config_from_dict(raw, dm.tokenizer.vocab_size, train_cfg), train_cfg, dm)


def main(argv=None) -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = parser.add_subparsers(dest="command", required=True)
    for name in ("train", "eval"):
        p = sub.add_parser(name)
        p.add_argument("--config", default="config/config.yml")
        p.add_argument("--model", default="standalone_tiny")
        p.add_argument("--output-dir")
        p.add_argument("--device")
        if name == "train":
            p.add_argument("--resume-from")
        else:
            p.add_argument("--checkpoint", required=True)
            p.add_argument("--predictions-jsonl")
            p.add_argument("--traces-jsonl")
    args = parser.parse_args(argv)
    if args.command == "train":
        build_trainer(args.config, args.output_dir, args.resume_from, args.device, args.model).train()
        return
    trainer = build_trainer(args.config, args.output_dir, args.checkpoint, args.device, args.model)
    traces = args.traces_jsonl or str(Path(trainer.trace_dir) / "eval_traces.jsonl")
    trainer.test(save_predictions=args.predictions_jsonl, save_traces=traces)


if __name__ == "__main__":
    main()
