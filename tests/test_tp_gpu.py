"""Tensor-parallel PRA Llama engine on 2 GPUs against the fp32 oracle (skipped with fewer GPUs).

Child processes, one per GPU, NVLS off; the collectives are this library's kernels on
plain peer loads / stores.  The last case makes one rank skip an all-reduce so the
peer's bounded wait runs out and reports an error status.
"""

import os
import tempfile
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _rendezvous_file() -> str:
    """A fresh path for a file-based process-group rendezvous: no TCP port for the ranks to race
    other processes for (a port picked free can be taken before rank 0 listens on it)."""
    return os.path.join(tempfile.mkdtemp(prefix="pra_pg_"), "store")


def _worker(rank, world, port, queue):
    os.environ.update(NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"file://{store}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    result = {"rank": rank}
    try:
        from pdattention_b200.inference.llama_engine import LlamaWeights, PRALlamaEngine
        from pdattention_b200.models.llama import PRALlamaReference, reference_step, tiny_llama
        from pdattention_b200.parallel.tp import TensorParallel

        torch.manual_seed(0)
        cfg = tiny_llama(head_dim=64, hidden_size=128, num_attention_heads=4, num_key_value_heads=2,
                         chunk_tokens=16, top_k_chunks=3)
        model = PRALlamaReference(cfg).eval()
        model.reset_parameters(seed=0, std=0.08)
        chunks = torch.randint(0, cfg.vocab_size, (10, 16))
        lengths = torch.tensor([16, 16, 11, 16, 16, 9, 16, 16, 16, 13])
        tp = TensorParallel()
        engine = PRALlamaEngine(LlamaWeights.from_reference(model, "cuda", rank, world), "cuda", tp=tp,
                                decode_split_keys=64)
        engine.build_memory(chunks, lengths, batch_chunks=4)
        spans = [(0, 10), (3, 8)]
        engine.set_namespace(torch.tensor([a for a, _ in spans]), torch.tensor([b for _, b in spans]))
        ids = torch.randint(0, cfg.vocab_size, (2, 18))
        plen = torch.tensor([18, 11])
        logits = engine.prefill(ids, plen, 3).float().cpu()
        ref_mem = model.encode_chunks(chunks, lengths)
        caches = [[[None, None] for _ in range(cfg.num_hidden_layers)] for _ in range(2)]
        cos = []
        for b in range(2):
            ref, _ = reference_step(model, ids[b, : int(plen[b])], caches[b], ref_mem, list(range(*spans[b])))
            cos.append(float(F.cosine_similarity(logits[b], ref[-1], dim=0)))
        for _ in range(2):
            tok = torch.randint(0, cfg.vocab_size, (2,), generator=torch.Generator().manual_seed(7))
            got = engine.decode_step(tok).float().cpu()
            for b in range(2):
                ref, _ = reference_step(model, tok[b: b + 1], caches[b], ref_mem, list(range(*spans[b])))
                cos.append(float(F.cosine_similarity(got[b], ref[-1], dim=0)))
        torch.cuda.synchronize()
        tp.check()
        result["cos"] = cos
        # the fused decode GEMM + all-reduce against fp32 partials summed by NCCL
        gen = torch.Generator(device="cuda").manual_seed(100 + rank)
        errs = []
        for m, n, k in ((64, 4096, 512), (5, 256, 1792), (33, 1024, 128)):
            x = torch.randn(m, k, device="cuda", generator=gen).bfloat16()
            w = (torch.randn(n, k, device="cuda", generator=gen) * 0.05).bfloat16()
            res = torch.randn(m, n, device="cuda", generator=torch.Generator(device="cuda").manual_seed(9)).bfloat16()
            got = tp.fused_gemm_allreduce(x, w, res).float()
            want = x.float() @ w.float().t()
            dist.all_reduce(want)
            want += res.float()
            errs.append(float((got - want).abs().max() / want.abs().max()))
        torch.cuda.synchronize()
        tp.check()
        result["fused_err"] = errs
        # the routing kernel with the candidate exchange fused in == local top-k + all-gather + merge
        from pdattention_b200.ops import _ext

        ext = _ext.require()
        C, D, k, per = 300, 64, 5, 150
        g = torch.Generator(device="cuda").manual_seed(55)
        gists_all = F.normalize(torch.randn(C, D, device="cuda", generator=g), dim=-1)
        query = torch.randn(6, D, device="cuda", generator=g)  # identical on both ranks
        c0 = rank * per
        local_gists = gists_all[c0: c0 + per].contiguous()
        scores = (F.normalize(query, dim=-1) @ local_gists.t()).contiguous()
        start = torch.tensor([0, 20, 0, 100, 140, 0], device="cuda")
        end = torch.tensor([300, 250, 10, 300, 160, 150], device="cuda")
        lo = (start - c0).clamp(0, per).to(torch.int32)
        hi = (end - c0).clamp(0, per).to(torch.int32)
        clen = torch.full((C,), 8, device="cuda", dtype=torch.int32)
        row0 = torch.arange(C, device="cuda", dtype=torch.int32) * 8
        same = True
        for _ in range(3):  # consecutive calls alternate the receive halves
            fused = tp.route_exchange(scores, query, local_gists, lo, hi, k, 32, 20, k * 8, c0, 1, clen, row0)
            cs, ci = ext.route_topk(scores, query, local_gists, lo, hi, clen, row0, k, 32, -1, 0, True, c0, 1, 1)
            merged = tp.all_gather_columns(torch.cat([cs, ci.view(torch.float32)], dim=1))
            want = ext.route_merge(merged, world, k, 20, clen, row0, k * 8, False)
            same = same and torch.equal(fused[1], want[1]) and torch.equal(fused[2], want[2])
            for r in range(6):
                n = int(want[1][r])
                same = same and torch.equal(fused[0][r, :n], want[0][r, :n])
        torch.cuda.synchronize()
        tp.check()
        result["route_exchange_equal"] = same
        # timeout: rank 1 skips one all-reduce; rank 0's wait must run out and report
        dist.barrier()
        tp.max_spins = 1 << 14
        if rank == 0:
            x = torch.randn(8, 64, device="cuda").bfloat16()
            w = torch.randn(16, 64, device="cuda").bfloat16()
            tp.gemm_allreduce(x, w, None)
            torch.cuda.synchronize()
            result["timeout_code"] = int(tp.error.item())
            tp.error.zero_()
        dist.barrier()
        if rank == 0:  # the fused kernel's per-tile wait runs out the same way
            x = torch.randn(8, 64, device="cuda").bfloat16()
            w = torch.randn(256, 64, device="cuda").bfloat16()
            tp.fused_gemm_allreduce(x, w, None)
            torch.cuda.synchronize()
            result["fused_timeout_code"] = int(tp.error.item())
            tp.error.zero_()
        dist.barrier()
        if rank == 0:  # and the fused routing exchange's per-row wait
            tp.route_exchange(scores, query, local_gists, lo, hi, k, 32, 20, k * 8, c0, 1, clen, row0)
            torch.cuda.synchronize()
            result["route_timeout_code"] = int(tp.error.item())
            tp.error.zero_()
        dist.barrier()
        tp.buffers.close()
    except Exception as error:
        import traceback

        result["error"] = traceback.format_exc()
    finally:
        queue.put(result)
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tensor_parallel_engine_two_gpus():
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    store = _rendezvous_file()
    procs = [ctx.Process(target=_worker, args=(r, world, store, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        item = queue.get(timeout=300)
        results[item["rank"]] = item
    for p in procs:
        p.join(timeout=60)
    for rank, item in results.items():
        assert "error" not in item, item["error"]
        assert min(item["cos"]) > 0.99, item["cos"]
        assert max(item["fused_err"]) < 2e-2, item["fused_err"]
        assert item["route_exchange_equal"]
    assert results[0]["timeout_code"] == 1
    assert results[0]["fused_timeout_code"] == 2
    assert results[0]["route_timeout_code"] == 1
