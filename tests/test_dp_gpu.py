"""Fused peer-memory data-parallel gradient reduction on 2 GPUs (skipped with fewer).

The ranks are child processes, one per GPU, with NVLS off; the kernel uses plain
peer loads and stores.  Both output modes run: the bf16 average written back in
place into the gradient buffers (equal to the fp32 average of the same rank order
rounded to bf16) and the fp32 average in a separate buffer.  The timeout case makes a rank skip one reduction so the
peer's bounded wait runs out: the kernel must return with an error status that the
host reads, and the context must stay usable.
"""

import os
import tempfile
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _rendezvous_file() -> str:
    """A fresh path for a file-based process-group rendezvous: no TCP port for the ranks to race
    other processes for (a port picked free can be taken before rank 0 listens on it)."""
    return os.path.join(tempfile.mkdtemp(prefix="pra_pg_"), "store")


def _worker(rank: int, world: int, store: str, queue, out_dtype: str = "bf16") -> None:
    os.environ.update(NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"file://{store}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    result = {"rank": rank}
    try:
        from pdattention_b200.config import TrainConfig
        from pdattention_b200.models.fastpath import prepare_model
        from pdattention_b200.parallel.dp import attach_data_parallel
        from pdattention_b200.smoke import tiny_config

        import tempfile
        from pathlib import Path

        from pdattention_b200.config import ResolverServiceConfig
        from pdattention_b200.pra_train import _pra_batch_step
        from pdattention_b200.smoke import tiny_batch

        tok, batch = tiny_batch(Path(tempfile.mkdtemp()))
        torch.manual_seed(0)
        model = prepare_model(tiny_config(tok.vocab_size), "cuda")  # the batch's ids fit the vocabulary
        rt = model._device_runtime
        opt = model.build_optimizer(TrainConfig(device="cuda", learning_rate=1e-3))
        reducer = attach_data_parallel(model, opt, world, "peer", overlap=True, out_dtype=out_dtype)
        exact = (lambda t: t.bfloat16().float()) if out_dtype == "bf16" else (lambda t: t)  # noqa: E731
        grad = rt.flat.grad
        # the slot views now alias the peer-visible buffer
        gw = rt.layers[0]["qkv"].gw
        result["aliased"] = grad.data_ptr() <= gw.data_ptr() < grad.data_ptr() + grad.numel() * 2
        gen = torch.Generator(device="cuda").manual_seed(100 + rank)
        grad.copy_(torch.randn(grad.shape, generator=gen, device="cuda").bfloat16())
        gathered = [torch.empty_like(grad) for _ in range(world)]
        dist.all_gather(gathered, grad)  # before the reduction: in place it overwrites grad
        expected = gathered[0].float()
        for t in gathered[1:]:
            expected = expected + t.float()
        expected = expected * (1.0 / world)
        out = reducer.reduce()
        torch.cuda.synchronize()
        reducer.check()
        result["max_err"] = float((out.float() - exact(expected)).abs().max())
        # a second reduction reuses the signal area (epochs increase)
        grad.copy_(2 * gathered[rank])
        out = reducer.reduce()
        torch.cuda.synchronize()
        reducer.check()
        result["max_err2"] = float((out.float() - exact(2 * expected)).abs().max())
        # one optimizer step through the reducer keeps the replicas identical
        opt.step()
        checksum = rt.flat.master.double().sum().reshape(1)
        sums = [torch.zeros_like(checksum) for _ in range(world)]
        dist.all_gather(sums, checksum)
        result["replicas_equal"] = all(float(s) == float(sums[0]) for s in sums)
        # overlapped pieces (the hooks the native backward calls: head, blocks top-down, then
        # the rest at the optimizer) give the same average
        result["hooked"] = reducer.overlap and rt.grad_hooks is reducer
        grad.copy_(torch.randn(grad.shape, generator=gen, device="cuda").bfloat16())
        dist.all_gather(gathered, grad)
        expected = sum(t.float() for t in gathered) * (1.0 / world)
        reducer.before_stack()
        for li in reversed(range(len(reducer.layer_ranges))):
            reducer.after_layer(li)
        out = reducer.reduce()
        torch.cuda.synchronize()
        reducer.check()
        result["max_err3"] = float((out.float() - exact(expected)).abs().max())
        # a real step through the native training stack (the hooks fire during its backward)
        opt.zero_grad()
        loss, _ = _pra_batch_step(model, batch, "cuda", tok, ResolverServiceConfig(), None)
        loss.backward()
        result["pieces"] = len(reducer.done)
        opt.step()
        torch.cuda.synchronize()
        reducer.check()
        checksum = rt.flat.master.double().sum().reshape(1)
        dist.all_gather(sums, checksum)
        result["replicas_equal2"] = all(float(s) == float(sums[0]) for s in sums)
        dist.barrier()
        # timeout: rank 1 skips one reduction; rank 0's bounded wait must run out
        reducer.max_spins = 1 << 14
        if rank == 0:
            reducer.reduce()
            torch.cuda.synchronize()
            result["timeout_code"] = int(reducer.error.item())
            reducer.error.zero_()
            result["context_usable"] = bool(torch.ones(4, device="cuda").sum().item() == 4)
        dist.barrier()
        reducer.close()
    except Exception as error:  # reported to the parent
        result["error"] = repr(error)
    finally:
        queue.put(result)
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("out_dtype", ["bf16", "fp32"])
def test_peer_gradient_allreduce_two_gpus(out_dtype):
    from pdattention_b200.ops import _ext

    if not _ext.available():
        pytest.skip("extension not built")
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    store = _rendezvous_file()
    procs = [ctx.Process(target=_worker, args=(r, world, store, queue, out_dtype)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        item = queue.get(timeout=300)
        results[item["rank"]] = item
    for p in procs:
        p.join(timeout=60)
    for rank, item in results.items():
        assert "error" not in item, item
        assert item["aliased"], item
        assert item["max_err"] < 1e-5, item
        assert item["max_err2"] < 1e-5, item
        assert item["replicas_equal"], item
        assert item["hooked"], item
        assert item["max_err3"] < 1e-5, item
        assert item["pieces"] == 1 + 2, item  # head + the tiny model's 2 blocks before the optimizer step
        assert item["replicas_equal2"], item
    assert results[0]["timeout_code"] == 1, results[0]
    assert results[0]["context_usable"]
