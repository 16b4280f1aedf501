"""Data parallel training on CPU with gloo ranks, and failure detection between ranks.

Two processes train the TinyGPT-PRA object path through the generic engine; gradients are
averaged every step, so the replicas stay identical.  In the failure case one rank raises
between steps; the survivor's next collective must end with an error (short process-group
timeout / closed connection) instead of hanging.
"""

import os
import tempfile

import pytest
import torch
import torch.multiprocessing as mp


def _rendezvous_file() -> str:
    """A fresh file-store path: no TCP port that a concurrently running test could take first."""
    return os.path.join(tempfile.mkdtemp(prefix="pra_pg_"), "store")


def _setup(rank, world, store, root):
    os.environ.update(PRA_INIT_METHOD=f"file://{store}", RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from pdattention_b200.parallel.dist import maybe_init_distributed

    maybe_init_distributed(backend="gloo", timeout_s=20)


def _train_worker(rank, world, store, root, queue):
    result = {"rank": rank}
    try:
        _setup(rank, world, store, root)
        import torch.distributed as dist

        from pdattention_b200.config import PRAConfig, TrainConfig
        from pdattention_b200.data import PRADataModule
        from pdattention_b200.models.tiny import TinyPRAModel
        from pdattention_b200.pra_train import train_pra_model

        torch.manual_seed(rank)  # different init on purpose: the engine must broadcast rank 0's weights
        dm = PRADataModule("stage0_synthetic_memory", root, batch_size=2, max_seq_len=64, rank=rank,
                           world_size=world).load()
        cfg = PRAConfig(vocab_size=dm.tokenizer.vocab_size, d_model=32, n_heads=4, n_layers=2, max_seq_len=64,
                        device="cpu", pra_layer_ids=(0, 1))
        tcfg = TrainConfig(output_dir=os.path.join(root, "out"), experiment_name="dp", device="cpu", epochs=1,
                           max_steps=3, batch_size=2, eval_every_steps=100, save_every_steps=100,
                           log_every_steps=1, use_tensorboard=False, save_metric_plots=False)
        model = TinyPRAModel(cfg)
        out = train_pra_model(cfg=cfg, train_config=tcfg, datamodule=dm, model=model)
        params = torch.cat([p.detach().reshape(-1) for p in out["model"].parameters()])
        gathered = [torch.zeros_like(params) for _ in range(world)]
        dist.all_gather(gathered, params)
        result["max_diff"] = float(max((g - gathered[0]).abs().max() for g in gathered))
        dist.destroy_process_group()
    except Exception as error:  # reported to the parent
        import traceback

        result["error"] = traceback.format_exc()
    queue.put(result)


def _failing_worker(rank, world, store, root, queue):
    result = {"rank": rank}
    try:
        _setup(rank, world, store, root)
        import torch.distributed as dist

        t = torch.ones(4)
        dist.all_reduce(t)  # step 1: both ranks take part
        if rank == 1:
            raise RuntimeError("injected failure on rank 1 between steps")
        dist.all_reduce(t)  # step 2: rank 1 is gone; this must fail, not hang
        result["completed"] = True
    except Exception as error:
        result["error"] = type(error).__name__ + ": " + str(error)[:200]
    queue.put(result)
    queue.close()
    queue.join_thread()  # the result is flushed before the process leaves
    os._exit(0)  # leave without a clean group teardown (the peer is gone)


def _run(target, root, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    store = _rendezvous_file()
    procs = [ctx.Process(target=target, args=(r, world, store, root, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        item = queue.get(timeout=timeout)
        results[item["rank"]] = item
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


@pytest.fixture
def stage_root(tmp_path):
    from pdattention_b200.data.generators import generate_synthetic

    generate_synthetic(tmp_path / "stage0_synthetic_memory", n=8)
    return str(tmp_path)


def test_gloo_data_parallel_keeps_replicas_identical(stage_root):
    results = _run(_train_worker, stage_root)
    for item in results.values():
        assert "error" not in item, item.get("error")
        assert item["max_diff"] == 0.0


def test_rank_failure_surfaces_as_error_not_hang(stage_root):
    results = _run(_failing_worker, stage_root)
    assert "injected failure" in results[1]["error"]
    assert "error" in results[0] and not results[0].get("completed"), results[0]
