"""Parameter / memory estimates for a resolved config dict (``config/model_size.py``)."""

from __future__ import annotations

DTYPE_BYTES = {"float32": 4, "fp32": 4, "float": 4, "float16": 2, "fp16": 2, "bfloat16": 2, "bf16": 2}


def bytes_to_mib(value: float) -> float:
    return float(value) / (1024 ** 2)


def _linear(i: int, o: int, bias: bool = True) -> int:
    return i * o + (o if bias else 0)


def _mlp(d: int) -> int:
    return _linear(d, 4 * d) + _linear(4 * d, d)


def vanilla_block_params(d: int) -> int:
    return (3 * d * d + 3 * d) + _linear(d, d) + _mlp(d) + 2 * 2 * d


def pra_block_params(d: int) -> int:
    return 5 * _linear(d, d) + _mlp(d) + 2 * 2 * d


def mixed_block_params(d: int) -> int:
    return (3 * d * d + 3 * d) + _linear(d, d) + 5 * _linear(d, d) + _mlp(d) + 3 * 2 * d


def estimate_model_size(cfg: dict, *, vocab_size: int = 128, batch_size: int | None = None, dtype: str = "float32",
                        optimizer: str = "adamw") -> dict:
    model, train = cfg["model"], cfg.get("train", {})
    d, layers = int(model["d_model"]), int(model["n_layers"])
    vanilla, mixed = int(model.get("n_vanilla_layers", 0)), int(model.get("n_mixed_layers", 0))
    pra = max(layers - vanilla - mixed, 0)
    seq = int(model["max_seq_len"])
    batch = int(batch_size if batch_size is not None else train.get("batch_size", 1))
    width = DTYPE_BYTES.get(dtype.lower())
    if width is None:
        raise ValueError(f"Unsupported dtype for size estimate: {dtype}")
    params = (vocab_size * d + seq * d + vanilla * vanilla_block_params(d) + mixed * mixed_block_params(d)
              + pra * pra_block_params(d) + 2 * d + d * vocab_size)
    p_bytes = params * width
    opt_bytes = params * width * (2 if optimizer.lower() in {"adam", "adamw"} else 0)
    act_bytes = batch * seq * d * width * max(layers, 1) * 2
    return {"selected_model": cfg.get("selected_model", "default"), "d_model": d, "n_layers": layers,
            "n_vanilla_layers": vanilla, "n_mixed_layers": mixed, "n_pra_layers": pra, "max_seq_len": seq,
            "batch_size": batch, "vocab_size": int(vocab_size), "dtype": dtype, "optimizer": optimizer,
            "total_params": int(params), "parameter_mib": bytes_to_mib(p_bytes), "gradient_mib": bytes_to_mib(p_bytes),
            "optimizer_state_mib": bytes_to_mib(opt_bytes), "activation_mib": bytes_to_mib(act_bytes),
            "inference_mib": bytes_to_mib(p_bytes + act_bytes),
            "training_mib": bytes_to_mib(2 * p_bytes + opt_bytes + act_bytes)}
