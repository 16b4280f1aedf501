"""The ``pra`` command line: ``train``, ``eval``, ``config show``, ``size``, ``dataset show``.

Flags, defaults and precedence follow ``src/pra_torch/cli.py``: built-in
defaults <- ``config/config.yml`` (working directory) <- ``-c`` file <-
``models.<name>`` profile (may set ``model`` / ``train`` / ``pra`` / ``resolver``
/ ``cache`` / ``standalone``) <- command-line flags (unset flags are dropped).
A missing config file warns and continues.  ``pra train`` additionally takes
``--nproc`` to launch data-parallel ranks (one per GPU, NCCL) on this node.
"""

from __future__ import annotations

import copy
import dataclasses
import os
import random
import subprocess
import sys
from pathlib import Path

import click
import torch
import yaml

from .config import CacheServiceConfig, PRAConfig, ResolverServiceConfig, TrainConfig, deep_update
from .config import read_yaml as read_yaml_file
from .data.datamodules import PRADataModule
from .data.datasets import read_jsonl
from .eval import run_evaluation
from .model_size import estimate_model_size
from .pra_train import train_pra_model
from .runtime.train import resolve_device

DEFAULT_CONFIG_PATH = Path("config") / "config.yml"
PACKAGED_CONFIG_PATH = Path(__file__).resolve().parents[1] / "config" / "config.yml"

_MODEL_KEYS = ("d_model", "n_heads", "n_layers", "n_vanilla_layers", "n_mixed_layers", "d_ff", "max_seq_len",
               "dropout", "model_variant")
_PRA_DEFAULT_KEYS = (
    "max_prompt_direct_tokens", "model_max_context_tokens", "prompt_overflow_mode", "max_prompt_gists",
    "max_materialized_memory_tokens", "context_safety_reserve_tokens", "pra_layer_ids", "top_k_references",
    "top_k_chunks_per_reference", "trigger_threshold", "memory_transport", "memory_alpha", "search_strategy",
    "routing_backend", "reference_score_aggregation", "reference_level_gist_mode", "reference_gists_per_reference",
    "reference_gist_score_aggregation", "gist_mode", "gists_per_chunk", "gist_score_aggregation",
    "max_gists_per_reference", "gist_overflow_policy", "chunking_mode", "fixed_chunk_tokens",
    "fixed_chunk_overlap_tokens", "encoding_chunking", "routing_chunking", "encoding_context_mode",
    "reference_overflow_policy", "detail_materialization", "kv_cache_residency", "kv_cache_pin_memory",
    "kv_cache_non_blocking", "memory_bucket_count", "memory_bucket_strategy", "cache_build_mode", "use_summary",
    "summary_mode", "recursive_refs_enabled", "recursive_max_depth", "recursive_max_total_references",
    "recursive_max_total_tokens", "recursive_max_children_per_reference", "recursive_cycle_policy",
    "recursive_missing_ref_policy",
)
# Every other PRAConfig field may also be set in the ``pra`` section of a YAML file.
_PRA_PASSTHROUGH = tuple(f.name for f in dataclasses.fields(PRAConfig)
                         if f.name not in {"vocab_size", "d_model", "n_heads", "n_layers", "n_vanilla_layers",
                                           "n_mixed_layers", "d_ff", "max_seq_len", "dropout", "model_variant",
                                           "pra_layer_ids", "top_k_references", "top_k_chunks_per_reference",
                                           "trigger_threshold", "memory_transport", "memory_alpha", "top_k_refs",
                                           "use_cross_attention_memory", "use_concat_memory", "batch_size", "lr",
                                           "steps", "device", "semantic_chunker"})


def _pra_defaults() -> dict:
    base = {f.name: f.default for f in dataclasses.fields(PRAConfig) if f.default is not dataclasses.MISSING}
    out = {k: base[k] for k in _PRA_DEFAULT_KEYS}
    out["pra_layer_ids"] = list(out["pra_layer_ids"])
    return out


BUILTIN_CONFIG = {
    "model": {"d_model": 128, "n_heads": 4, "n_layers": 4, "n_vanilla_layers": 0, "n_mixed_layers": 0, "d_ff": None,
              "max_seq_len": 96, "dropout": 0.0},
    "pra": _pra_defaults(),
    "train": {"steps": 300, "batch_size": 8, "lr": 3e-4, "device": "auto", "out": "pra_tiny.pt",
              "dataset_stage": "stage0_synthetic_memory", "data_dir": "data", "max_examples": None, "shuffle": True,
              "num_workers": 0, "pin_memory": False, "persistent_workers": False},
    "resolver": {"type": "in_memory", "options": {}},
    "cache": {"type": "simple", "options": {}},
    "eval": {"ckpt": "pra_tiny.pt", "device": "auto", "examples": 20, "dataset_stage": "stage0_synthetic_memory",
             "data_dir": "data", "max_examples": None, "max_new_tokens": 24, "seed": 0, "batch_size": 8,
             "num_workers": 0, "pin_memory": False, "persistent_workers": False},
}


def read_yaml(path: Path) -> dict:
    if not path.exists():
        click.echo(f"Warning: config file not found: {path}", err=True)
        return {}
    return read_yaml_file(path)


def apply_named_model(cfg: dict, model_name: str = "default") -> dict:
    profile = (cfg.get("models") or {}).get(model_name)
    if profile is None:
        if model_name == "default":
            return cfg
        raise KeyError(f"Unknown model profile: {model_name}")
    profile = copy.deepcopy(profile)
    direct = {k: profile.pop(k) for k in list(profile) if k in cfg["model"]}
    if "model" in profile:
        deep_update(cfg["model"], profile["model"] or {})
    deep_update(cfg["model"], direct)
    for section in ("train", "pra", "resolver", "cache", "standalone"):
        if section in profile:
            deep_update(cfg.setdefault(section, {}), profile[section] or {})
    cfg["selected_model"] = model_name
    return cfg


def load_config(config_path: str | None = None, model_name: str = "default") -> dict:
    cfg = copy.deepcopy(BUILTIN_CONFIG)
    local = DEFAULT_CONFIG_PATH
    if not local.exists() and PACKAGED_CONFIG_PATH.exists():
        local = PACKAGED_CONFIG_PATH
    deep_update(cfg, read_yaml(local))
    if config_path:
        deep_update(cfg, read_yaml(Path(config_path)))
    return apply_named_model(cfg, model_name)


def parse_layer_ids(value) -> tuple[int, ...]:
    if value is None:
        return tuple()
    if isinstance(value, str):
        return tuple(int(p.strip()) for p in value.split(",") if p.strip())
    return tuple(int(v) for v in value)


def command_overrides(values: dict) -> dict:
    return {k: v for k, v in values.items() if v is not None}


def model_kwargs(cfg: dict) -> dict:
    model, pra = cfg["model"], cfg["pra"]
    out = {
        "d_model": int(model["d_model"]), "n_heads": int(model["n_heads"]), "n_layers": int(model["n_layers"]),
        "n_vanilla_layers": int(model.get("n_vanilla_layers", 0)),
        "n_mixed_layers": int(model.get("n_mixed_layers", 0)),
        "d_ff": int(model["d_ff"]) if model.get("d_ff") is not None else None,
        "max_seq_len": int(model["max_seq_len"]), "dropout": float(model["dropout"]),
        "model_variant": str(model.get("model_variant", "custom")),
        "pra_layer_ids": parse_layer_ids(pra["pra_layer_ids"]),
        "top_k_references": int(pra["top_k_references"]),
        "top_k_chunks_per_reference": int(pra["top_k_chunks_per_reference"]),
        "trigger_threshold": float(pra["trigger_threshold"]),
        "memory_transport": str(pra.get("memory_transport", "native_kv")),
        "memory_alpha": float(pra["memory_alpha"]),
    }
    out.update({k: pra[k] for k in ("use_cross_attention_memory", "use_concat_memory") if pra.get(k) is not None})
    out.update({k: pra[k] for k in _PRA_PASSTHROUGH if k in pra})
    return out


def build_pra_config(cfg: dict, *, vocab_size: int, batch_size: int, lr: float, steps: int, device: str) -> PRAConfig:
    return PRAConfig(vocab_size=vocab_size, batch_size=batch_size, lr=lr, steps=steps, device=device,
                     **model_kwargs(cfg))


def apply_service_overrides(cfg: dict, options: dict) -> None:
    given = command_overrides(options)
    if "resolver_type" in given:
        cfg["resolver"]["type"] = given["resolver_type"]
    if "cache_type" in given:
        cfg["cache"]["type"] = given["cache_type"]


_PRA_FLAG_KEYS = {"pra_layer_ids", "top_k_references", "top_k_chunks_per_reference", "trigger_threshold",
                  "memory_transport", "use_cross_attention_memory", "use_concat_memory", "memory_alpha"}


def apply_common_overrides(cfg: dict, options: dict) -> None:
    for key, value in command_overrides(options).items():
        if key in _MODEL_KEYS:
            cfg["model"][key] = value
        elif key in _PRA_FLAG_KEYS:
            cfg["pra"][key] = parse_layer_ids(value) if key == "pra_layer_ids" else value


def _stack(options):
    def wrap(func):
        for option in reversed(options):
            func = option(func)
        return func

    return wrap


common_model_options = _stack([
    click.option("-M", "--d-model", type=int), click.option("-H", "--n-heads", type=int),
    click.option("-L", "--n-layers", type=int), click.option("-V", "--n-vanilla-layers", type=int),
    click.option("-Y", "--n-mixed-layers", type=int), click.option("-l", "--max-seq-len", type=int),
    click.option("-p", "--dropout", type=float),
    click.option("-P", "--pra-layer-ids", type=str, help="Comma-separated layer ids, e.g. 2,3."),
    click.option("-k", "--top-k-references", "--top-k-refs", type=int),
    click.option("--top-k-chunks-per-reference", type=int), click.option("-t", "--trigger-threshold", type=float),
    click.option("--memory-transport", type=click.Choice(["native_kv", "cross_attention"])),
    click.option("-x/-X", "--use-cross-attention-memory/--no-use-cross-attention-memory", default=None),
    click.option("-u/-U", "--use-concat-memory/--no-use-concat-memory", default=None),
    click.option("-a", "--memory-alpha", type=float),
])
common_service_options = _stack([click.option("-R", "--resolver-type", type=str),
                                 click.option("-A", "--cache-type", type=str)])


@click.group()
def cli():
    """PRA command line (B200 build)."""


def _launch_ranks(nproc: int) -> None:
    """Re-run this command under ``torch.distributed.run`` with one rank per GPU."""
    argv = [a for a in sys.argv[1:] if not a.startswith("--nproc")]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
           "--master-addr=127.0.0.1", "--master-port=29531", "-m", "pdattention_b200.cli", *argv]
    raise SystemExit(subprocess.call(cmd, env={**os.environ, "PRA_LAUNCHED": "1"}))


@cli.command()
@click.option("-c", "--config", "config_path", type=click.Path(dir_okay=False))
@click.option("--model", "model_name", default="default", show_default=True,
              help="Named model profile from the models section.")
@click.option("-s", "--steps", type=int)
@click.option("-b", "--batch-size", type=int)
@click.option("-r", "--lr", type=float)
@click.option("-d", "--device", type=str)
@click.option("-o", "--out", type=str)
@click.option("-g", "--dataset-stage", type=str)
@click.option("-D", "--data-dir", type=str)
@click.option("-m", "--max-examples", type=int)
@click.option("-w", "--num-workers", type=int)
@click.option("-i/-I", "--pin-memory/--no-pin-memory", default=None)
@click.option("-W/-N", "--persistent-workers/--no-persistent-workers", default=None)
@click.option("-q/-Q", "--shuffle/--no-shuffle", default=None)
@click.option("--nproc", type=int, default=None, help="Data-parallel ranks on this node (one per GPU).")
@common_service_options
@common_model_options
def train(config_path, model_name, nproc, **options):
    """Train TinyPRA."""
    if nproc and nproc > 1 and os.environ.get("PRA_LAUNCHED") != "1":
        _launch_ranks(nproc)
    try:
        cfg = load_config(config_path, model_name=model_name)
    except KeyError as exc:
        raise click.ClickException(str(exc)) from exc
    apply_common_overrides(cfg, options)
    apply_service_overrides(cfg, options)
    tcfg = cfg["train"]
    for key, value in command_overrides(options).items():
        if key in tcfg:
            tcfg[key] = value
    from .parallel.dist import maybe_init_distributed

    rank, world = maybe_init_distributed()
    device = resolve_device(tcfg["device"])
    if device == "cuda" and world > 1:
        device = f"cuda:{torch.cuda.current_device()}"
    datamodule = PRADataModule(dataset_stage=tcfg["dataset_stage"], data_dir=tcfg["data_dir"],
                               max_examples=tcfg["max_examples"], batch_size=int(tcfg["batch_size"]),
                               max_seq_len=int(cfg["model"]["max_seq_len"]), shuffle=bool(tcfg["shuffle"]),
                               num_workers=int(tcfg["num_workers"]), pin_memory=bool(tcfg["pin_memory"]),
                               persistent_workers=bool(tcfg["persistent_workers"]), rank=rank, world_size=world).load()
    pra_cfg = build_pra_config(cfg, vocab_size=datamodule.tokenizer.vocab_size, batch_size=int(tcfg["batch_size"]),
                               lr=float(tcfg["lr"]), steps=int(tcfg["steps"]), device=device)
    out = Path(tcfg["out"])
    steps = int(tcfg["steps"])
    runtime = TrainConfig(
        experiment_name=out.stem, output_dir=str(out.parent if out.parent != Path(".") else "out"), device=device,
        epochs=1, max_steps=steps if steps > 0 else None, batch_size=int(tcfg["batch_size"]), grad_accum_steps=1,
        learning_rate=float(tcfg["lr"]), max_seq_len=int(cfg["model"]["max_seq_len"]),
        num_workers=int(tcfg["num_workers"]), pin_memory=bool(tcfg["pin_memory"]),
        persistent_workers=bool(tcfg["persistent_workers"]), dataset_stage=tcfg["dataset_stage"],
        data_dir=tcfg["data_dir"], max_examples=tcfg["max_examples"], shuffle=bool(tcfg["shuffle"]),
        eval_every_steps=max(steps + 1, 1), save_every_steps=max(steps + 1, 1), log_every_steps=1,
        use_tensorboard=False, resolver_config=ResolverServiceConfig.from_value(cfg["resolver"]),
        cache_config=CacheServiceConfig.from_value(cfg["cache"]))
    from .models.fastpath import prepare_model

    model = prepare_model(pra_cfg, device)
    result = train_pra_model(cfg=pra_cfg, train_config=runtime, datamodule=datamodule, model=model,
                             resolver_config=runtime.resolver_config, cache_config=runtime.cache_config)
    if rank == 0:
        torch.save({"model": result["model"].state_dict(), "cfg": pra_cfg.__dict__, "stoi": datamodule.tokenizer.stoi,
                    "itos": datamodule.tokenizer.itos, "dataset_stage": tcfg["dataset_stage"],
                    "resolver_config": runtime.resolver_config.__dict__, "cache_config": runtime.cache_config.__dict__},
                   tcfg["out"])
        click.echo(f"saved {tcfg['out']}")


@cli.command(name="eval")
@click.option("-c", "--config", "config_path", type=click.Path(dir_okay=False))
@click.option("-K", "--ckpt", type=str)
@click.option("-d", "--device", type=str)
@click.option("-e", "--examples", type=int)
@click.option("-g", "--dataset-stage", type=str)
@click.option("-D", "--data-dir", type=str)
@click.option("-m", "--max-examples", type=int)
@click.option("-n", "--max-new-tokens", type=int)
@click.option("-S", "--seed", type=int)
@click.option("-b", "--batch-size", type=int)
@click.option("-w", "--num-workers", type=int)
@click.option("-i/-I", "--pin-memory/--no-pin-memory", default=None)
@click.option("-W/-N", "--persistent-workers/--no-persistent-workers", default=None)
@common_service_options
@common_model_options
def eval(config_path, **options):  # noqa: A001 - command name is part of the CLI
    """Evaluate TinyPRA baselines."""
    cfg = load_config(config_path)
    apply_common_overrides(cfg, options)
    apply_service_overrides(cfg, options)
    ecfg = cfg["eval"]
    for key, value in command_overrides(options).items():
        if key in ecfg:
            ecfg[key] = value
    random.seed(int(ecfg["seed"]))
    torch.manual_seed(int(ecfg["seed"]))
    limit = ecfg["max_examples"] if ecfg["max_examples"] is not None else ecfg["examples"]
    datamodule = PRADataModule(dataset_stage=ecfg["dataset_stage"], data_dir=ecfg["data_dir"], max_examples=limit,
                               batch_size=int(ecfg["batch_size"]), max_seq_len=int(cfg["model"]["max_seq_len"]),
                               shuffle=False, num_workers=int(ecfg["num_workers"]), pin_memory=bool(ecfg["pin_memory"]),
                               persistent_workers=bool(ecfg["persistent_workers"])).load()
    kwargs = model_kwargs(cfg)
    kwargs.pop("max_seq_len")
    run_evaluation(ckpt=ecfg["ckpt"], device=resolve_device(ecfg["device"]), datamodule=datamodule,
                   max_new_tokens=int(ecfg["max_new_tokens"]), max_seq_len=int(cfg["model"]["max_seq_len"]),
                   resolver_config=ResolverServiceConfig.from_value(cfg["resolver"]),
                   cache_config=CacheServiceConfig.from_value(cfg["cache"]), **kwargs)


@cli.group()
def config():
    """Inspect CLI configuration."""


@config.command(name="show")
@click.option("-c", "--config", "config_path", type=click.Path(dir_okay=False))
def config_show(config_path):
    """Show merged default configuration."""
    click.echo(yaml.safe_dump(load_config(config_path), sort_keys=False))


@cli.command()
@click.option("-c", "--config", "config_path", type=click.Path(dir_okay=False))
@click.option("--model", "model_name", default="default", show_default=True,
              help="Named model profile from the models section.")
@click.option("-v", "--vocab-size", type=int, default=128, show_default=True)
@click.option("-b", "--batch-size", type=int)
@click.option("-d", "--dtype", type=click.Choice(["float32", "fp32", "float16", "fp16", "bfloat16", "bf16"]),
              default="float32", show_default=True)
@click.option("-o", "--optimizer", type=click.Choice(["adamw", "adam", "sgd", "none"]), default="adamw",
              show_default=True)
def size(config_path, model_name, vocab_size, batch_size, dtype, optimizer):
    """Estimate memory requirements for a named model profile."""
    try:
        cfg = load_config(config_path, model_name=model_name)
    except KeyError as exc:
        raise click.ClickException(str(exc)) from exc
    click.echo(yaml.safe_dump(estimate_model_size(cfg, vocab_size=vocab_size, batch_size=batch_size, dtype=dtype,
                                                  optimizer=optimizer), sort_keys=False))


@cli.group()
def dataset():
    """Inspect datasets."""


@dataset.command(name="show")
@click.option("-c", "--config", "config_path", type=click.Path(dir_okay=False))
@click.option("-g", "--dataset-stage", type=str)
@click.option("-D", "--data-dir", type=str)
@click.option("-m", "--max-examples", type=int)
def dataset_show(config_path, dataset_stage, data_dir, max_examples):
    """Show stats for a named dataset stage."""
    cfg = load_config(config_path)
    stage = dataset_stage or cfg["train"]["dataset_stage"]
    root = data_dir or cfg["train"]["data_dir"]
    path = Path(root) / stage
    module = PRADataModule(stage, root, max_examples=max_examples, shuffle=False).load()
    stats = {"stage": stage, "data_dir": str(root), "documents": len(read_jsonl(path / "documents.jsonl")),
             "references": len(read_jsonl(path / "references.jsonl")),
             "questions": len(read_jsonl(path / "questions.jsonl")), "loaded_examples": len(module.dataset),
             "expected_refs": sum(len(s.target_reference_ids) for s in module.dataset),
             "expected_anchors": sum(len(s.metadata.get("expected_anchors", [])) for s in module.dataset)}
    click.echo(yaml.safe_dump(stats, sort_keys=False))


@dataset.command(name="generate")
@click.option("-g", "--dataset-stage", type=str, required=True)
@click.option("-D", "--data-dir", type=str, default="data", show_default=True)
@click.option("-n", "--examples", type=int, default=64, show_default=True)
@click.option("-S", "--seed", type=int, default=0, show_default=True)
def dataset_generate(dataset_stage, data_dir, examples, seed):
    """Write a synthetic stage (kv QA, hierarchical tokens, or a demo stage)."""
    from .data.datasets import dataset_class_for_stage
    from .data import generators

    target = Path(data_dir) / dataset_stage
    if dataset_stage == "synthetic_hierarchical_tokens":
        generators.generate_hierarchical_tokens(target, examples=examples, seed=seed)
    else:
        name = dataset_class_for_stage(dataset_stage).generator_name
        getattr(generators, name)(target, n=examples, seed=seed)
    click.echo(f"wrote {target}")


if __name__ == "__main__":
    cli()
