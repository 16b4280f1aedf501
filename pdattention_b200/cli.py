"""The ``pra`` command line: ``train``, ``eval``, ``config show``, ``size``, ``dataset show|generate``.

Configuration is a stack of layers, later layers winning key by key
(``src/pra_torch/cli.py:23-170`` defines the same order and the same flags):

1. built-in defaults (``BUILTIN_CONFIG``);
2. ``config/config.yml`` from the working directory (else the packaged copy);
3. the ``-c`` file (a missing file prints a warning and is skipped);
4. the ``models.<name>`` profile chosen with ``--model``: top-level model keys and
   its ``model`` / ``train`` / ``pra`` / ``resolver`` / ``cache`` / ``standalone``
   sections;
5. command-line flags that were given (unset flags leave the stack alone).

``pra train --nproc N`` relaunches itself under ``torch.distributed.run`` with
one data-parallel rank per GPU of this node.
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
PROFILE_SECTIONS = ("train", "pra", "resolver", "cache", "standalone")

# ``model`` section keys (architecture) and the PRAConfig fields that are architecture or
# flag-driven; every other PRAConfig field may be set in the ``pra`` section.
_MODEL_KEYS = ("d_model", "n_heads", "n_layers", "n_vanilla_layers", "n_mixed_layers", "d_ff", "max_seq_len",
               "dropout", "model_variant")
_PRA_FLAGS = ("pra_layer_ids", "top_k_references", "top_k_chunks_per_reference", "trigger_threshold",
              "memory_transport", "use_cross_attention_memory", "use_concat_memory", "memory_alpha")
_NOT_FROM_PRA_SECTION = {*_MODEL_KEYS, *_PRA_FLAGS, "vocab_size", "top_k_refs", "batch_size", "lr", "steps",
                         "device", "semantic_chunker"}
_PRA_PASSTHROUGH = tuple(f.name for f in dataclasses.fields(PRAConfig) if f.name not in _NOT_FROM_PRA_SECTION)
# PRAConfig defaults shown by ``pra config show`` under ``pra``.
_PRA_SHOWN = ("max_prompt_direct_tokens", "model_max_context_tokens", "prompt_overflow_mode", "max_prompt_gists",
              "max_materialized_memory_tokens", "context_safety_reserve_tokens", "pra_layer_ids", "top_k_references",
              "top_k_chunks_per_reference", "trigger_threshold", "memory_transport", "memory_alpha",
              "search_strategy", "routing_backend", "reference_score_aggregation", "reference_level_gist_mode",
              "reference_gists_per_reference", "reference_gist_score_aggregation", "gist_mode", "gists_per_chunk",
              "gist_score_aggregation", "max_gists_per_reference", "gist_overflow_policy", "chunking_mode",
              "fixed_chunk_tokens", "fixed_chunk_overlap_tokens", "encoding_chunking", "routing_chunking",
              "encoding_context_mode", "reference_overflow_policy", "detail_materialization", "kv_cache_residency",
              "kv_cache_pin_memory", "kv_cache_non_blocking", "memory_bucket_count", "memory_bucket_strategy",
              "cache_build_mode", "use_summary", "summary_mode", "recursive_refs_enabled", "recursive_max_depth",
              "recursive_max_total_references", "recursive_max_total_tokens", "recursive_max_children_per_reference",
              "recursive_cycle_policy", "recursive_missing_ref_policy")


def _pra_defaults() -> dict:
    defaults = {f.name: f.default for f in dataclasses.fields(PRAConfig) if f.default is not dataclasses.MISSING}
    shown = {name: defaults[name] for name in _PRA_SHOWN}
    shown["pra_layer_ids"] = list(shown["pra_layer_ids"])
    return shown


_LOADER = {"num_workers": 0, "pin_memory": False, "persistent_workers": False}
BUILTIN_CONFIG = {
    "model": {"d_model": 128, "n_heads": 4, "n_layers": 4, "n_vanilla_layers": 0, "n_mixed_layers": 0, "d_ff": None,
              "max_seq_len": 96, "dropout": 0.0},
    "pra": _pra_defaults(),
    "train": {"steps": 300, "batch_size": 8, "lr": 3e-4, "device": "auto", "out": "pra_tiny.pt",
              "dataset_stage": "stage0_synthetic_memory", "data_dir": "data", "max_examples": None, "shuffle": True,
              **_LOADER},
    "resolver": {"type": "in_memory", "options": {}},
    "cache": {"type": "simple", "options": {}},
    "eval": {"ckpt": "pra_tiny.pt", "device": "auto", "examples": 20, "dataset_stage": "stage0_synthetic_memory",
             "data_dir": "data", "max_examples": None, "max_new_tokens": 24, "seed": 0, "batch_size": 8, **_LOADER},
}


# -- the configuration stack ---------------------------------------------------------------
def read_yaml(path: Path) -> dict:
    """A YAML layer, or an empty one (with a warning on stderr) when the file is missing."""
    if Path(path).exists():
        return read_yaml_file(path)
    click.echo(f"Warning: config file not found: {path}", err=True)
    return {}


def apply_named_model(cfg: dict, model_name: str = "default") -> dict:
    """Layer the ``models.<model_name>`` profile onto ``cfg`` (in place; returns it)."""
    profile = (cfg.get("models") or {}).get(model_name)
    if profile is None:
        if model_name != "default":
            raise KeyError(f"Unknown model profile: {model_name}")
        return cfg
    profile = copy.deepcopy(profile)
    top_level = {key: profile.pop(key) for key in list(profile) if key in cfg["model"]}
    for layer in (profile.get("model") or {}, top_level):  # the profile's model section, then bare keys
        deep_update(cfg["model"], layer)
    for section in PROFILE_SECTIONS:
        if section in profile:
            deep_update(cfg.setdefault(section, {}), profile[section] or {})
    cfg["selected_model"] = model_name
    return cfg


def load_config(config_path: str | None = None, model_name: str = "default") -> dict:
    """Layers 1-4 of the stack (flags are applied by each command)."""
    layers = [DEFAULT_CONFIG_PATH if DEFAULT_CONFIG_PATH.exists() or not PACKAGED_CONFIG_PATH.exists()
              else PACKAGED_CONFIG_PATH]
    if config_path:
        layers.append(Path(config_path))
    cfg = copy.deepcopy(BUILTIN_CONFIG)
    for path in layers:
        deep_update(cfg, read_yaml(path))
    return apply_named_model(cfg, model_name)


def parse_layer_ids(value) -> tuple[int, ...]:
    """``"2,3"`` / ``[2, 3]`` / ``None`` -> ``(2, 3)`` / ``(2, 3)`` / ``()``."""
    if value is None:
        return ()
    parts = value.split(",") if isinstance(value, str) else value
    return tuple(int(str(p).strip()) for p in parts if str(p).strip())


def command_overrides(values: dict) -> dict:
    """The flags that were actually given."""
    return {key: value for key, value in values.items() if value is not None}


def apply_common_overrides(cfg: dict, options: dict) -> None:
    """Model and PRA flags into their sections."""
    for key, value in command_overrides(options).items():
        if key in _MODEL_KEYS:
            cfg["model"][key] = value
        elif key in _PRA_FLAGS:
            cfg["pra"][key] = parse_layer_ids(value) if key == "pra_layer_ids" else value


def apply_service_overrides(cfg: dict, options: dict) -> None:
    """``-R`` / ``-A`` select the resolver and cache service types."""
    given = command_overrides(options)
    for flag, section in (("resolver_type", "resolver"), ("cache_type", "cache")):
        if flag in given:
            cfg[section]["type"] = given[flag]


def _apply_section_overrides(section: dict, options: dict) -> None:
    section.update({k: v for k, v in command_overrides(options).items() if k in section})


# -- configuration -> PRAConfig ------------------------------------------------------------
def _int_or_none(value):
    return None if value is None else int(value)


_MODEL_CASTS = {"d_model": int, "n_heads": int, "n_layers": int, "max_seq_len": int, "dropout": float}
_PRA_CASTS = {"top_k_references": int, "top_k_chunks_per_reference": int, "trigger_threshold": float,
              "memory_alpha": float}


def model_kwargs(cfg: dict) -> dict:
    """PRAConfig keyword arguments of a resolved configuration (without vocabulary / run fields)."""
    model, pra = cfg["model"], cfg["pra"]
    kwargs = {key: cast(model[key]) for key, cast in _MODEL_CASTS.items()}
    kwargs.update(n_vanilla_layers=int(model.get("n_vanilla_layers", 0)),
                  n_mixed_layers=int(model.get("n_mixed_layers", 0)), d_ff=_int_or_none(model.get("d_ff")),
                  model_variant=str(model.get("model_variant", "custom")))
    kwargs.update({key: cast(pra[key]) for key, cast in _PRA_CASTS.items()})
    kwargs["pra_layer_ids"] = parse_layer_ids(pra["pra_layer_ids"])
    kwargs["memory_transport"] = str(pra.get("memory_transport", "native_kv"))
    kwargs.update({key: pra[key] for key in ("use_cross_attention_memory", "use_concat_memory")
                   if pra.get(key) is not None})
    kwargs.update({key: pra[key] for key in _PRA_PASSTHROUGH if key in pra})
    return kwargs


def build_pra_config(cfg: dict, *, vocab_size: int, batch_size: int, lr: float, steps: int, device: str) -> PRAConfig:
    return PRAConfig(vocab_size=vocab_size, batch_size=batch_size, lr=lr, steps=steps, device=device,
                     **model_kwargs(cfg))


# -- flags ----------------------------------------------------------------------------------
def _options(specs):
    """One decorator applying click options given as (args, kwargs) pairs, first spec outermost."""
    def decorate(func):
        for args, kwargs in reversed(specs):
            func = click.option(*args, **kwargs)(func)
        return func

    return decorate


def _switch(short, long):
    return (short, long), {"default": None}


common_model_options = _options([
    (("-M", "--d-model"), {"type": int}), (("-H", "--n-heads"), {"type": int}),
    (("-L", "--n-layers"), {"type": int}), (("-V", "--n-vanilla-layers"), {"type": int}),
    (("-Y", "--n-mixed-layers"), {"type": int}), (("-l", "--max-seq-len"), {"type": int}),
    (("-p", "--dropout"), {"type": float}),
    (("-P", "--pra-layer-ids"), {"type": str, "help": "Comma-separated layer ids, e.g. 2,3."}),
    (("-k", "--top-k-references", "--top-k-refs"), {"type": int}),
    (("--top-k-chunks-per-reference",), {"type": int}), (("-t", "--trigger-threshold"), {"type": float}),
    (("--memory-transport",), {"type": click.Choice(["native_kv", "cross_attention"])}),
    _switch("-x/-X", "--use-cross-attention-memory/--no-use-cross-attention-memory"),
    _switch("-u/-U", "--use-concat-memory/--no-use-concat-memory"),
    (("-a", "--memory-alpha"), {"type": float}),
])
common_service_options = _options([(("-R", "--resolver-type"), {"type": str}), (("-A", "--cache-type"), {"type": str})])
_loader_options = _options([
    (("-w", "--num-workers"), {"type": int}), _switch("-i/-I", "--pin-memory/--no-pin-memory"),
    _switch("-W/-N", "--persistent-workers/--no-persistent-workers")])
_config_option = click.option("-c", "--config", "config_path", type=click.Path(dir_okay=False))
_profile_option = click.option("--model", "model_name", default="default", show_default=True,
                               help="Named model profile from the models section.")


@click.group()
def cli():
    """PRA command line (B200 build)."""


def _relaunch_per_gpu(nproc: int) -> None:
    """Run this command again under ``torch.distributed.run``, one rank per GPU."""
    argv = [arg for arg in sys.argv[1:] if not arg.startswith("--nproc")]
    launcher = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
                "--master-addr=127.0.0.1", "--master-port=29531", "-m", "pdattention_b200.cli"]
    raise SystemExit(subprocess.call(launcher + argv, env={**os.environ, "PRA_LAUNCHED": "1"}))


def _resolved(config_path, model_name, options) -> dict:
    try:
        cfg = load_config(config_path, model_name=model_name)
    except KeyError as exc:
        raise click.ClickException(str(exc)) from exc
    apply_common_overrides(cfg, options)
    apply_service_overrides(cfg, options)
    return cfg


def _datamodule(section: dict, cfg: dict, **extra) -> PRADataModule:
    return PRADataModule(dataset_stage=section["dataset_stage"], data_dir=section["data_dir"],
                         batch_size=int(section["batch_size"]), max_seq_len=int(cfg["model"]["max_seq_len"]),
                         num_workers=int(section["num_workers"]), pin_memory=bool(section["pin_memory"]),
                         persistent_workers=bool(section["persistent_workers"]), **extra).load()


def _services(cfg: dict) -> tuple[ResolverServiceConfig, CacheServiceConfig]:
    return ResolverServiceConfig.from_value(cfg["resolver"]), CacheServiceConfig.from_value(cfg["cache"])


@cli.command()
@_config_option
@_profile_option
@_options([(("-s", "--steps"), {"type": int}), (("-b", "--batch-size"), {"type": int}), (("-r", "--lr"), {"type": float}),
           (("-d", "--device"), {"type": str}), (("-o", "--out"), {"type": str}),
           (("-g", "--dataset-stage"), {"type": str}), (("-D", "--data-dir"), {"type": str}),
           (("-m", "--max-examples"), {"type": int})])
@_loader_options
@_options([_switch("-q/-Q", "--shuffle/--no-shuffle"),
           (("--nproc",), {"type": int, "default": None, "help": "Data-parallel ranks on this node (one per GPU)."})])
@common_service_options
@common_model_options
def train(config_path, model_name, nproc, **options):
    """Train TinyPRA."""
    if nproc and nproc > 1 and os.environ.get("PRA_LAUNCHED") != "1":
        _relaunch_per_gpu(nproc)
    cfg = _resolved(config_path, model_name, options)
    run = cfg["train"]
    _apply_section_overrides(run, options)
    from .parallel.dist import maybe_init_distributed

    rank, world = maybe_init_distributed()
    device = resolve_device(run["device"])
    if device == "cuda" and world > 1:
        device = f"cuda:{torch.cuda.current_device()}"
    data = _datamodule(run, cfg, max_examples=run["max_examples"], shuffle=bool(run["shuffle"]), rank=rank,
                       world_size=world)
    steps, batch = int(run["steps"]), int(run["batch_size"])
    pra_cfg = build_pra_config(cfg, vocab_size=data.tokenizer.vocab_size, batch_size=batch, lr=float(run["lr"]),
                               steps=steps, device=device)
    out = Path(run["out"])
    resolver, cache = _services(cfg)
    never = max(steps + 1, 1)  # one run of `steps` optimizer updates, no mid-run validation or checkpoint
    engine = TrainConfig(
        experiment_name=out.stem, output_dir=str(out.parent if out.parent != Path(".") else "out"), device=device,
        epochs=1, max_steps=steps if steps > 0 else None, batch_size=batch, grad_accum_steps=1,
        learning_rate=float(run["lr"]), max_seq_len=int(cfg["model"]["max_seq_len"]),
        num_workers=int(run["num_workers"]), pin_memory=bool(run["pin_memory"]),
        persistent_workers=bool(run["persistent_workers"]), dataset_stage=run["dataset_stage"],
        data_dir=run["data_dir"], max_examples=run["max_examples"], shuffle=bool(run["shuffle"]),
        eval_every_steps=never, save_every_steps=never, log_every_steps=1, use_tensorboard=False,
        resolver_config=resolver, cache_config=cache)
    from .models.fastpath import prepare_model

    result = train_pra_model(cfg=pra_cfg, train_config=engine, datamodule=data, model=prepare_model(pra_cfg, device),
                             resolver_config=resolver, cache_config=cache)
    if rank == 0:  # the pra_tiny.pt payload
        torch.save({"model": result["model"].state_dict(), "cfg": pra_cfg.__dict__, "stoi": data.tokenizer.stoi,
                    "itos": data.tokenizer.itos, "dataset_stage": run["dataset_stage"],
                    "resolver_config": resolver.__dict__, "cache_config": cache.__dict__}, run["out"])
        click.echo(f"saved {run['out']}")


@cli.command(name="eval")
@_config_option
@_options([(("-K", "--ckpt"), {"type": str}), (("-d", "--device"), {"type": str}), (("-e", "--examples"), {"type": int}),
           (("-g", "--dataset-stage"), {"type": str}), (("-D", "--data-dir"), {"type": str}),
           (("-m", "--max-examples"), {"type": int}), (("-n", "--max-new-tokens"), {"type": int}),
           (("-S", "--seed"), {"type": int}), (("-b", "--batch-size"), {"type": int})])
@_loader_options
@common_service_options
@common_model_options
def eval(config_path, **options):  # noqa: A001 - command name is part of the CLI
    """Evaluate TinyPRA baselines."""
    cfg = _resolved(config_path, "default", options)
    section = cfg["eval"]
    _apply_section_overrides(section, options)
    seed = int(section["seed"])
    random.seed(seed)
    torch.manual_seed(seed)
    limit = section["max_examples"] if section["max_examples"] is not None else section["examples"]
    data = _datamodule(section, cfg, max_examples=limit, shuffle=False)
    kwargs = model_kwargs(cfg)
    kwargs.pop("max_seq_len")
    resolver, cache = _services(cfg)
    run_evaluation(ckpt=section["ckpt"], device=resolve_device(section["device"]), datamodule=data,
                   max_new_tokens=int(section["max_new_tokens"]), max_seq_len=int(cfg["model"]["max_seq_len"]),
                   resolver_config=resolver, cache_config=cache, **kwargs)


@cli.group()
def config():
    """Inspect CLI configuration."""


@config.command(name="show")
@_config_option
def config_show(config_path):
    """Show merged default configuration."""
    click.echo(yaml.safe_dump(load_config(config_path), sort_keys=False))


@cli.command()
@_config_option
@_profile_option
@click.option("-v", "--vocab-size", type=int, default=128, show_default=True)
@click.option("-b", "--batch-size", type=int)
@click.option("-d", "--dtype", type=click.Choice(["float32", "fp32", "float16", "fp16", "bfloat16", "bf16"]),
              default="float32", show_default=True)
@click.option("-o", "--optimizer", type=click.Choice(["adamw", "adam", "sgd", "none"]), default="adamw",
              show_default=True)
def size(config_path, model_name, vocab_size, batch_size, dtype, optimizer):
    """Estimate memory requirements for a named model profile."""
    cfg = _resolved(config_path, model_name, {})
    click.echo(yaml.safe_dump(estimate_model_size(cfg, vocab_size=vocab_size, batch_size=batch_size, dtype=dtype,
                                                  optimizer=optimizer), sort_keys=False))


@cli.group()
def dataset():
    """Inspect datasets."""


@dataset.command(name="show")
@_config_option
@click.option("-g", "--dataset-stage", type=str)
@click.option("-D", "--data-dir", type=str)
@click.option("-m", "--max-examples", type=int)
def dataset_show(config_path, dataset_stage, data_dir, max_examples):
    """Show stats for a named dataset stage."""
    cfg = load_config(config_path)
    stage = dataset_stage or cfg["train"]["dataset_stage"]
    root = data_dir or cfg["train"]["data_dir"]
    loaded = PRADataModule(stage, root, max_examples=max_examples, shuffle=False).load().dataset
    counts = {name: len(read_jsonl(Path(root) / stage / f"{name}.jsonl"))
              for name in ("documents", "references", "questions")}
    stats = {"stage": stage, "data_dir": str(root), **counts, "loaded_examples": len(loaded),
             "expected_refs": sum(len(s.target_reference_ids) for s in loaded),
             "expected_anchors": sum(len(s.metadata.get("expected_anchors", [])) for s in loaded)}
    click.echo(yaml.safe_dump(stats, sort_keys=False))


@dataset.command(name="generate")
@click.option("-g", "--dataset-stage", type=str, required=True)
@click.option("-D", "--data-dir", type=str, default="data", show_default=True)
@click.option("-n", "--examples", type=int, default=64, show_default=True)
@click.option("-S", "--seed", type=int, default=0, show_default=True)
def dataset_generate(dataset_stage, data_dir, examples, seed):
    """Write a synthetic stage (kv QA, hierarchical tokens, or a demo stage)."""
    from .data import generators
    from .data.datasets import dataset_class_for_stage

    target = Path(data_dir) / dataset_stage
    if dataset_stage == "synthetic_hierarchical_tokens":
        generators.generate_hierarchical_tokens(target, examples=examples, seed=seed)
    else:
        getattr(generators, dataset_class_for_stage(dataset_stage).generator_name)(target, n=examples, seed=seed)
    click.echo(f"wrote {target}")


if __name__ == "__main__":
    cli()
