"""The ``pra`` command line and its configuration stack (the reference's CLI behaviour)."""

from click.testing import CliRunner

from pdattention_b200.cli import apply_named_model, cli, load_config, model_kwargs


def test_config_show_uses_default_yaml():
    result = CliRunner().invoke(cli, ["config", "show"])
    assert result.exit_code == 0
    assert "stage0_synthetic_memory" in result.output and "model:" in result.output


def test_missing_config_warns_and_uses_defaults():
    result = CliRunner().invoke(cli, ["config", "show", "-c", "missing.yml"])
    assert result.exit_code == 0
    assert "Warning: config file not found: missing.yml" in result.output
    assert "stage0_synthetic_memory" in result.output


def test_yaml_layer_then_named_profile(tmp_path):
    path = tmp_path / "models.yml"
    path.write_text("model:\n  d_model: 128\n  n_heads: 4\ntrain:\n  batch_size: 8\n  steps: 7\npra:\n"
                    "  top_k_references: 2\nmodels:\n  small:\n    d_model: 32\n    model:\n      d_model: 48\n"
                    "      n_layers: 3\n    train:\n      batch_size: 2\n    pra:\n      top_k_references: 1\n",
                    encoding="utf-8")
    cfg = load_config(str(path), model_name="small")
    assert cfg["selected_model"] == "small"
    assert cfg["model"]["d_model"] == 32  # a bare profile key beats the profile's model section
    assert cfg["model"]["n_layers"] == 3 and cfg["model"]["n_heads"] == 4
    assert cfg["train"]["batch_size"] == 2 and cfg["train"]["steps"] == 7
    assert cfg["pra"]["top_k_references"] == 1


def test_default_profile_falls_back_and_unknown_profile_fails():
    cfg = {"model": {"d_model": 128}, "models": {"small": {"d_model": 32}}}
    assert apply_named_model(cfg, "default")["model"]["d_model"] == 128
    result = CliRunner().invoke(cli, ["size", "--model", "no_such_profile"])
    assert result.exit_code != 0 and "Unknown model profile" in result.output


def test_central_profiles_and_gist_defaults():
    tiny = load_config(model_name="standalone_tiny")
    assert (tiny["model"]["d_model"], tiny["model"]["n_layers"], tiny["pra"]["pra_layer_ids"]) == (32, 2, [0, 1])
    assert tiny["standalone"]["experiment_name"] == "standalone_tiny"
    kwargs = model_kwargs(load_config())
    assert (kwargs["gists_per_chunk"], kwargs["gist_mode"], kwargs["memory_transport"]) == (1, "mean", "native_kv")
    assert kwargs["prompt_overflow_mode"] == "truncate" and kwargs["max_prompt_gists"] is None
    mixed = load_config(model_name="tdx_pra_tiny")
    assert mixed["model"]["model_variant"] == "tdx_pra" and mixed["model"]["n_vanilla_layers"] == 2
