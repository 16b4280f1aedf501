"""Systems benchmarks (routing speed, index reuse, K/V residency, batch forward): data on CPU,
one tiny run of each on the GPU."""

import tempfile
from pathlib import Path

import pytest
import torch

from pdattention_b200 import benchmarks


def test_lookup_examples_have_one_evidence_unit_first():
    examples = benchmarks.lookup_examples(3, units=255)
    for ex in examples:
        assert len(ex.source_units) == 255 and ex.source_units[0].is_evidence
        assert sum(u.is_evidence for u in ex.source_units) == 1
        assert ex.question.split()[0] == ex.source_units[0].text.split("=")[0]
        assert ex.answer == ex.source_units[0].text.split("=")[1]
    assert benchmarks.lookup_examples(3)[1].source_units == examples[1].source_units  # seeded


def test_loader_splits_the_source_into_references(tmp_path):
    from pdattention_b200.data import WordIdTokenizer

    batches = benchmarks._loader(Path(tmp_path), 64, 2, WordIdTokenizer(8000))
    assert len(batches) == 2
    assert batches[0]["input_ids"].shape[0] == 1


@pytest.mark.gpu
def test_each_suite_runs_on_the_device(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    rows = benchmarks.routing_speed(tiers=("tiny",), splits=(32,), examples=2, root=Path(tmp_path) / "a")
    by = {r["routing_backend"]: r for r in rows}
    assert set(by) == {"legacy", "tensorized", "device"}
    assert by["device"]["routing_latency_seconds"] > 0 and by["device"]["retrieved_physical_kv_tokens"] > 0
    rows = benchmarks.kv_residency(tiers=("tiny",), splits=(32,), examples=2, warm_repeats=2,
                                   root=Path(tmp_path) / "b")
    gpu, cpu = (next(r for r in rows if r["kv_cache_residency"] == k) for k in ("gpu", "cpu"))
    assert cpu["gpu_cached_kv_bytes"] == 0 < cpu["selected_kv_transfer_bytes"]
    assert gpu["cached_kv_bytes"] == cpu["cached_kv_bytes"] > 0
    rows = benchmarks.routing_index_reuse(tiers=("tiny",), splits=(32,), examples=2, root=Path(tmp_path) / "c")
    assert rows[0]["tensorized_warm_index_ms"] > 0
    rows = benchmarks.batch_forward(batch_sizes=(1, 4), repeats=1, tier="tiny", root=Path(tmp_path) / "d")
    assert [r["batch_size"] for r in rows] == [1, 4] and rows[1]["batched_prompt_seconds"] > 0
