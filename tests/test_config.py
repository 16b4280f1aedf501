import dataclasses

import pytest

from pdattention_b200.config import PRAConfig, TrainConfig, deep_update


def test_field_names_and_defaults_match_reference(ref):
    mine = {f.name: f.default for f in dataclasses.fields(PRAConfig)}
    theirs = {f.name: f.default for f in dataclasses.fields(ref.config.PRAConfig)}
    assert mine.keys() == theirs.keys()
    assert {k: v for k, v in mine.items() if v is not dataclasses.MISSING} == \
        {k: v for k, v in theirs.items() if v is not dataclasses.MISSING}


@pytest.mark.parametrize("kwargs", [
    {}, {"model_variant": "td_pra", "n_layers": 6}, {"model_variant": "tdx_pra", "n_layers": 5},
    {"model_variant": "td_sa"}, {"max_seq_len": 64, "model_max_context_tokens": 48, "context_safety_reserve_tokens": 8},
    {"top_k_refs": 3}, {"use_cross_attention_memory": True}, {"use_concat_memory": True},
    {"chunking_mode": "fixed", "fixed_chunk_tokens": 16, "chunk_overlap_fraction": 0.25},
    {"routing_chunking": {"mode": "fixed", "chunk_tokens": 8}},
])
def test_normalisation_matches_reference(ref, kwargs):
    with _maybe_warn():
        mine = PRAConfig(**kwargs)
        theirs = ref.config.PRAConfig(**kwargs)
    for f in dataclasses.fields(PRAConfig):
        a, b = getattr(mine, f.name), getattr(theirs, f.name)
        if dataclasses.is_dataclass(a):
            a, b = dataclasses.asdict(a), dataclasses.asdict(b)
        assert a == b, f.name
    assert mine.effective_prompt_direct_tokens == theirs.effective_prompt_direct_tokens
    assert mine.effective_model_max_context_tokens == theirs.effective_model_max_context_tokens
    assert mine.resolved_chunk_overlap_tokens == theirs.resolved_chunk_overlap_tokens


class _maybe_warn:
    def __enter__(self):
        import warnings

        self._ctx = warnings.catch_warnings()
        self._ctx.__enter__()
        warnings.simplefilter("ignore")

    def __exit__(self, *exc):
        return self._ctx.__exit__(*exc)


@pytest.mark.parametrize("kwargs", [
    {"max_seq_len": 0}, {"model_max_context_tokens": 200, "max_seq_len": 100}, {"top_k_references": -1},
    {"gist_mode": "bogus"}, {"search_strategy": "x"}, {"fixed_chunk_overlap_tokens": 64},
    {"chunk_overlap_fraction": 0.2, "fixed_chunk_overlap_tokens": 2}, {"kv_cache_residency": "cpu",
                                                                       "cache_build_mode": "trainable_gist"},
    {"n_vanilla_layers": 3, "n_mixed_layers": 3, "n_layers": 4}, {"reference_level_gist_mode": "ref_end"},
    {"gist_som_init": "grid"}, {"chunk_iou_threshold": 2.0}, {"recursive_max_depth": -1},
])
def test_invalid_configs_rejected_like_reference(ref, kwargs):
    with pytest.raises((ValueError, NotImplementedError)):
        ref.config.PRAConfig(**kwargs)
    with pytest.raises((ValueError, NotImplementedError)):
        PRAConfig(**kwargs)


def test_prompt_tail_offset():
    cfg = PRAConfig(max_seq_len=64, prompt_position_mode="historical")
    assert cfg.prompt_tail_position_offset(20, 30) == 20
    assert cfg.prompt_tail_position_offset(40, 30) == 0
    assert PRAConfig(max_seq_len=64).prompt_tail_position_offset(20, 30) == 0


def test_train_config_services_and_validation():
    cfg = TrainConfig(resolver_config="in_memory", cache_config={"type": "paged", "options": {}})
    assert cfg.resolver_config.type == "in_memory" and cfg.cache_config.type == "paged"
    with pytest.raises(ValueError):
        TrainConfig(batch_size=0)


def test_deep_update_merges_nested():
    base = {"a": {"b": 1, "c": 2}, "d": 3}
    deep_update(base, {"a": {"b": 5}, "e": 1})
    assert base == {"a": {"b": 5, "c": 2}, "d": 3, "e": 1}


def test_every_named_profile_runs_on_the_device_path_except_head_dim_8():
    """Every ``models.*`` profile of config/config.yml maps onto the device path (vanilla / mixed
    blocks, dropout, the tiny head widths); only ``standalone_tiny`` (d_model 32 over 4 heads:
    head width 8, below the tensor-core fragment) keeps the object path."""
    from pathlib import Path

    from pdattention_b200.cli import build_pra_config, load_config, read_yaml
    from pdattention_b200.models.fastpath import unsupported_reason

    path = Path(__file__).resolve().parents[1] / "config" / "config.yml"
    names = sorted(read_yaml(path)["models"])
    reasons = {}
    for name in names:
        cfg = build_pra_config(load_config(str(path), name), vocab_size=512, batch_size=2, lr=1e-3, steps=1,
                               device="cuda")
        reasons[name] = unsupported_reason(cfg)
    assert reasons.pop("standalone_tiny") == "head_dim=8"
    assert all(reason is None for reason in reasons.values()), reasons
