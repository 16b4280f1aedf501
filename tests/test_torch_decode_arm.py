"""The plain-PyTorch decode comparison arm (baseline/torch_pra_decode.py) on a tiny model, on CPU."""

import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "baseline"))
import torch_pra_decode  # noqa: E402

TINY = dict(hidden=64, heads=4, kv_heads=2, head_dim=16, inter=128, layers=2, vocab=97, rope_theta=10000.0, eps=1e-5)


def test_memory_routing_prefill_and_decode():
    model = torch_pra_decode.TorchPRALlama(TINY, "cpu", top_k=2)
    chunks = torch.randint(0, 97, (6, 64), generator=torch.Generator().manual_seed(0))
    model.build_memory(chunks, batch=4)
    assert model.gists.shape == (2, 6, 32)
    assert torch.allclose(model.gists.norm(dim=-1), torch.ones(2, 6), atol=1e-5)
    prompts = torch.randint(0, 97, (3, 10), generator=torch.Generator().manual_seed(1))
    tok = model.prefill(prompts, max_new=4, row_batch=2)
    assert tok.shape == (3,)
    steps = [tok]
    for _ in range(3):
        steps.append(model.decode_step(steps[-1]))
    assert model.length == 13 and all(int(t.max()) < 97 for t in steps)
    # routing picks the top-2 chunks by cosine of the group-mean pre-rotary query
    q = torch.randn(3, 4, 16)  # 4 query heads in 2 KV groups
    ids = model._route(0, q)
    rq = torch.nn.functional.normalize(q.float().unflatten(1, (2, 2)).mean(2).flatten(1), dim=-1)
    want = (rq @ model.gists[0].t()).topk(2).indices
    assert torch.equal(ids, want)


def test_namespaces_and_position_offsets():
    model = torch_pra_decode.TorchPRALlama(TINY, "cpu", top_k=2)
    chunks = torch.randint(0, 97, (8, 64), generator=torch.Generator().manual_seed(2))
    model.build_memory(chunks, batch=8)
    model.ns = (torch.tensor([0, 4]), torch.tensor([4, 8]))  # row 0 owns chunks 0-3, row 1 chunks 4-7
    model.pos_offset = torch.tensor([100, 0])
    model._rows = torch.arange(2)
    ids = model._route(1, torch.randn(2, 4, 16))
    assert bool((ids[0] < 4).all()) and bool((ids[1] >= 4).all())
    tok = model.prefill(torch.randint(0, 97, (2, 6), generator=torch.Generator().manual_seed(3)), max_new=3)
    nxt = model.decode_step(tok)
    assert nxt.shape == (2,) and model.length == 7
    # row 0's cached keys were rotated at positions 100.., row 1's at 0..: the same token's key differs
    k_row0, k_row1 = model.cache_k[0, 0, 0], model.cache_k[0, 1, 0]
    assert k_row0.shape == k_row1.shape
