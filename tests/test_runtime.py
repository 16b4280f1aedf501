import json
import warnings

import pytest
import torch
from click.testing import CliRunner

from pdattention_b200.cli import cli
from pdattention_b200.config import PRAConfig, TrainConfig
from pdattention_b200.data import PRADataModule
from pdattention_b200.data.generators import generate_hierarchy, generate_synthetic
from pdattention_b200.memory import (CacheBuildState, InMemoryResolver, PRASimpleMemoryCache,
                                     RecursiveReferenceCacheBuilder, ResolutionBudget, ResolutionBudgetExceeded)
from pdattention_b200.models import TinyPRAModel
from pdattention_b200.runtime import CheckpointError, read_checkpoint
from pdattention_b200.trainer import PRAStandaloneTrainer


@pytest.fixture
def data_root(tmp_path):
    generate_synthetic(tmp_path / "data" / "stage0_synthetic_memory", n=6)
    generate_hierarchy(tmp_path / "data" / "stage1_hierarchical_synthetic", n=3)
    return tmp_path


def _trainer(root, **kw):
    dm = PRADataModule("stage0_synthetic_memory", str(root / "data"), batch_size=2, max_seq_len=64).load()
    cfg = PRAConfig(vocab_size=dm.tokenizer.vocab_size, d_model=32, n_heads=4, n_layers=2, max_seq_len=64,
                    device="cpu", pra_layer_ids=(0, 1))
    tcfg = TrainConfig(output_dir=str(root / "out"), experiment_name="t", device="cpu", epochs=1, batch_size=2,
                       eval_every_steps=2, save_every_steps=2, log_every_steps=1, use_tensorboard=False,
                       save_metric_plots=False, **kw)
    return PRAStandaloneTrainer(cfg, tcfg, dm)


def test_trainer_trains_checkpoints_and_resumes(data_root):
    trainer = _trainer(data_root)
    result = trainer.train()
    assert "test_loss" in result and trainer.global_step > 0
    latest = trainer.checkpoint.latest_path
    payload = read_checkpoint(latest)
    for key in ("model", "optimizer", "scheduler", "config", "epoch", "global_step", "cfg", "stoi", "itos",
                "reference_vocabulary", "tokenizer_type"):
        assert key in payload
    again = _trainer(data_root, resume_from=str(latest))
    assert again.global_step == trainer.global_step
    preds, traces = data_root / "p.jsonl", data_root / "t.jsonl"
    again.test(save_predictions=str(preds), save_traces=str(traces))
    rows = [json.loads(line) for line in traces.read_text().splitlines()]
    assert rows and "selected_chunks_by_layer" in rows[0] and "routing_configuration" in rows[0]
    metrics = json.loads((data_root / "out" / "t" / "metrics.json").read_text())
    assert any(r["split"] == "train_batch" for r in metrics["records"])


def test_corrupt_checkpoint_is_reported(tmp_path):
    bad = tmp_path / "latest.pt"
    bad.write_bytes(b"not a checkpoint")
    with pytest.raises(CheckpointError):
        read_checkpoint(bad)


def _builder(docs, **kw):
    cfg = PRAConfig(vocab_size=200, d_model=16, n_heads=2, n_layers=2, max_seq_len=128, recursive_refs_enabled=True,
                    **kw)
    from pdattention_b200.data import PRATokenizer

    tok = PRATokenizer([d["text"] if isinstance(d, dict) else d for d in docs.values()])
    cache = PRASimpleMemoryCache()
    return RecursiveReferenceCacheBuilder(TinyPRAModel(cfg), InMemoryResolver(docs), tok, cache, cfg), cache


def test_recursion_cycle_missing_budget_and_failure_policies():
    docs = {"a": {"text": "A <REF_1>", "reference_table": {"<REF_1>": "b"}},
            "b": {"text": "B <REF_1> <REF_2>", "reference_table": {"<REF_1>": "a", "<REF_2>": "zzz"}}}
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        builder, cache = _builder(docs)
        builder.ensure_cached("a")
    kinds = [(e.uri, e.event) for e in builder.events]
    assert ("a", "cycle") in kinds and ("zzz", "missing") in kinds and cache.has("a") and cache.has("b")
    builder, _ = _builder(docs, recursive_cycle_policy="error", recursive_missing_ref_policy="skip")
    with pytest.raises(RuntimeError):
        builder.ensure_cached("a")
    assert builder.cache.state("a") == CacheBuildState.FAILED
    budget = ResolutionBudget(max_total_references=1, max_total_tokens=10)
    budget.consume(5)
    with pytest.raises(ResolutionBudgetExceeded):
        budget.consume(1)


def test_resolver_failure_marks_failed_and_reraises():
    class Exploding(InMemoryResolver):
        def resolve(self, uri, summary_only=False):
            if uri == "b":
                raise RuntimeError("backend down")
            return super().resolve(uri, summary_only)

    docs = {"a": {"text": "A <REF_1>", "reference_table": {"<REF_1>": "b"}}, "b": "B"}
    builder, cache = _builder(docs)
    builder.resolver = Exploding(docs)
    with pytest.raises(RuntimeError):
        builder.ensure_cached("a")
    assert cache.state("a") == CacheBuildState.FAILED and "backend down" in cache.failure("a")


def test_cli_commands(data_root, monkeypatch):
    monkeypatch.chdir(data_root)
    runner = CliRunner()
    out = runner.invoke(cli, ["config", "show"])
    assert out.exit_code == 0 and "pra:" in out.output
    out = runner.invoke(cli, ["size", "--model", "td_pra_gpt2_small", "-v", "50257"])
    assert out.exit_code == 0 and "total_params" in out.output
    out = runner.invoke(cli, ["dataset", "show", "-g", "stage1_hierarchical_synthetic", "-D", "data"])
    assert out.exit_code == 0 and "questions: 3" in out.output
    out = runner.invoke(cli, ["train", "--model", "standalone_tiny", "-s", "2", "-b", "2", "-d", "cpu", "-o",
                              "out/tiny.pt", "-D", "data"])
    assert out.exit_code == 0, out.output
    ckpt = torch.load(data_root / "out" / "tiny.pt", weights_only=False)
    assert {"model", "cfg", "stoi", "itos", "dataset_stage", "resolver_config", "cache_config"} <= set(ckpt)
    out = runner.invoke(cli, ["eval", "-K", "out/tiny.pt", "-d", "cpu", "-D", "data", "-e", "3", "-n", "2", "-l", "64"])
    assert out.exit_code == 0 and "PRA eval report (checkpoint)" in out.output
    out = runner.invoke(cli, ["train", "--model", "missing_profile"])
    assert out.exit_code != 0


def test_flat_grad_rehome_keeps_views_aliased():
    """Moving the flat gradient into another buffer re-points every slot view in place."""
    from pdattention_b200.models.fastpath import FlatParams
    from pdattention_b200.models.tiny import TinyPRAModel
    from pdattention_b200.smoke import tiny_config

    model = TinyPRAModel(tiny_config(64))
    flat = FlatParams(model, 128)
    flat.grad.copy_(torch.arange(flat.grad.numel()).to(torch.bfloat16))
    views = [flat.view(flat.grad, "blocks.0.attn.o_proj.weight"), flat.view(flat.grad, "token_emb.weight")]
    before = [v.clone() for v in views]
    new = torch.zeros(flat.grad.numel() + 64, dtype=torch.bfloat16)[64:]
    flat.rehome_grad(new, views)
    assert flat.grad is new
    for v, b in zip(views, before):
        assert torch.equal(v, b)
        assert new.data_ptr() <= v.data_ptr() < new.data_ptr() + new.numel() * 2
    views[0].fill_(3)
    start = flat.offsets["blocks.0.attn.o_proj.weight"]
    assert float(new[start]) == 3.0


def test_standalone_entry_points_train_and_eval(data_root):
    """``python -m pdattention_b200.standalone train|eval`` with a YAML like the packaged one."""
    import yaml

    from pdattention_b200.standalone import build_trainer, main

    cfg = {"model": {"d_model": 32, "n_heads": 4, "n_layers": 2},
           "pra": {"pra_layer_ids": [0, 1], "trigger_threshold": 0.0},
           "standalone": {"experiment_name": "sa", "output_dir": str(data_root / "out"), "device": "cpu",
                          "epochs": 1, "batch_size": 2, "eval_every_steps": 2, "save_every_steps": 2,
                          "log_every_steps": 1, "use_tensorboard": False, "save_metric_plots": False,
                          "max_examples": 4, "max_seq_len": 64, "dataset_stage": "stage0_synthetic_memory",
                          "data_dir": str(data_root / "data")}}
    path = data_root / "sa.yml"
    path.write_text(yaml.safe_dump(cfg))
    trainer = build_trainer(str(path), model_name="default")
    assert trainer.model.cfg.d_model == 32 and trainer.model.cfg.pra_layer_ids == (0, 1)
    main(["train", "--config", str(path), "--model", "default"])
    ckpt = data_root / "out" / "sa" / "checkpoints" / "latest.pt"
    assert ckpt.exists()
    traces = data_root / "sa_traces.jsonl"
    main(["eval", "--config", str(path), "--model", "default", "--checkpoint", str(ckpt),
          "--traces-jsonl", str(traces)])
    assert traces.read_text().strip()


def test_reduction_ranges_tile_the_flat_gradient():
    """The overlapped gradient reduction's pieces: one contiguous range per block holding
    exactly that block's parameters, in layout order, and the LM head's range last; the
    embeddings and final norm are what the optimizer-time reduction covers."""
    from pdattention_b200.models import TinyPRAModel
    from pdattention_b200.models.fastpath import FlatParams
    from pdattention_b200.parallel.dp import reduction_ranges
    from pdattention_b200.smoke import tiny_config

    cfg = tiny_config(96)
    cfg.device = "cpu"
    model = TinyPRAModel(cfg)
    flat = FlatParams(model, (cfg.vocab_size + 127) // 128 * 128)
    layers, head = reduction_ranges(flat)
    assert len(layers) == cfg.n_layers
    for i, (start, count) in enumerate(layers):
        assert start % 8 == 0 and count % 8 == 0 and count > 0
        inside = [n for n, off in flat.offsets.items() if start <= off < start + count]
        assert inside and all(n.startswith(f"blocks.{i}.") for n in inside)
        assert {n for n in flat.offsets if n.startswith(f"blocks.{i}.")} == set(inside)
        if i:
            assert start == layers[i - 1][0] + layers[i - 1][1]
    assert head == (flat.offsets["head.weight"], flat.total - flat.offsets["head.weight"])
    covered = sum(c for _, c in layers) + head[1]
    rest = [n for n, off in flat.offsets.items()
            if not any(s <= off < s + c for s, c in layers + [head])]
    assert set(rest) == {"token_emb.weight", "pos_emb.weight", "ln.weight", "ln.bias"}
    assert covered < flat.total


def test_planning_without_chunk_texts_keeps_plans():
    """Row planning decodes no chunk texts for fixed windows (the device path keeps only token
    ids and positions); the plans must equal those planned with the plain tokenizer."""
    import tempfile
    import types
    from pathlib import Path

    from pdattention_b200.config import ResolverServiceConfig
    from pdattention_b200.models import TinyPRAModel
    from pdattention_b200.models import fastpath
    from pdattention_b200.smoke import tiny_batch, tiny_config

    tok, batch = tiny_batch(Path(tempfile.mkdtemp()))
    cfg = tiny_config(tok.vocab_size)
    cfg.device = "cpu"
    assert cfg.chunking_mode == "fixed"
    model = TinyPRAModel(cfg)
    ctx = types.SimpleNamespace(cfg=model.cfg, model=model)
    resolver = ResolverServiceConfig()
    for item in batch["metadata"]:
        fast = fastpath.DeviceRuntime.plan_row(ctx, item, tok, resolver)
        original = fastpath._IdsOnlyTokenizer
        fastpath._IdsOnlyTokenizer = lambda t: t  # plain tokenizer: chunk texts decoded
        try:
            plain = fastpath.DeviceRuntime.plan_row(ctx, item, tok, resolver)
        finally:
            fastpath._IdsOnlyTokenizer = original
        assert [(e.uri, e.wave, e.visible, e.chunks) for e in fast.entries] == \
            [(e.uri, e.wave, e.visible, e.chunks) for e in plain.entries]
        assert [(c.chunk_id, c.token_start, c.token_end, c.token_ids, c.metadata) for c in fast.chunks] == \
            [(c.chunk_id, c.token_start, c.token_end, c.token_ids, c.metadata) for c in plain.chunks]
