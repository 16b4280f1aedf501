"""PRA Llama-family kernels and engine on the GPU against fp32 PyTorch / the fp32 oracle."""

import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ext():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from pdattention_b200.ops import _ext

    return _ext.require()


def test_rope_copy_and_silu_mul(ext):
    from pdattention_b200.models.llama import apply_rope, rope_tables, tiny_llama

    cfg = tiny_llama(head_dim=64)
    torch.manual_seed(0)
    M, H = 37, 3
    x = torch.randn(M, H * 64, device="cuda").bfloat16()
    pos = torch.randint(0, 500, (M,), device="cuda", dtype=torch.int32)
    half = 32
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, half, dtype=torch.float64) / half))
    ang = torch.arange(600, dtype=torch.float64)[:, None] * inv[None]
    cos_t, sin_t = ang.cos().float().cuda(), ang.sin().float().cuda()
    out = torch.empty(2 * M, H * 64, device="cuda").bfloat16()
    rows = (torch.arange(M, device="cuda", dtype=torch.int32) * 2 + 1)
    ext.rope_copy(x, out, rows, pos, cos_t, sin_t, H, 64)
    c, s = rope_tables(cfg, pos[None].cpu().long())
    ref = apply_rope(x.float().cpu().view(1, M, H, 64), c, s).view(M, H * 64)
    assert torch.allclose(out[1::2].float().cpu(), ref, atol=2e-2, rtol=2e-2)
    gu = torch.randn(M, 2 * 96, device="cuda").bfloat16()
    act = torch.empty(M, 96, device="cuda").bfloat16()
    ext.silu_mul(gu, act)
    g, u = gu.float()[:, :96], gu.float()[:, 96:]
    assert torch.allclose(act.float(), F.silu(g) * u, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("head_dim", [64, 128])
def test_decode_attention_matches_softmax(ext, head_dim):
    torch.manual_seed(1)
    B, H, Hkv, max_len = 3, 8, 2, 300
    q = torch.randn(B, H * head_dim, device="cuda").bfloat16()
    pool = torch.randn(500, 2 * Hkv * head_dim, device="cuda").bfloat16()
    mk, mv = pool[:, : Hkv * head_dim], pool[:, Hkv * head_dim:]
    mem_len = torch.tensor([70, 0, 130], device="cuda", dtype=torch.int32)
    mem_idx = torch.randint(0, 500, (B, 130), device="cuda", dtype=torch.int32)
    cache = torch.randn(2, B, max_len, Hkv * head_dim, device="cuda").bfloat16()
    loc_len = torch.tensor([5, 300, 129], device="cuda", dtype=torch.int32)
    out, eo, eml = ext.decode_attention(q, H, Hkv, head_dim, mk, mv, mem_idx, mem_len, cache[0], cache[1], loc_len,
                                        130 + max_len, 128, True)
    g = H // Hkv
    for b in range(B):
        n_m, n_l = int(mem_len[b]), int(loc_len[b])
        keys = torch.cat([mk[mem_idx[b, :n_m].long()], cache[0, b, :n_l]]).float().view(-1, Hkv, head_dim)
        vals = torch.cat([mv[mem_idx[b, :n_m].long()], cache[1, b, :n_l]]).float().view(-1, Hkv, head_dim)
        qb = q[b].float().view(H, head_dim)
        s = torch.einsum("hd,khd->hk", qb, keys.repeat_interleave(g, 1)) / math.sqrt(head_dim)
        ref = torch.einsum("hk,khd->hd", torch.softmax(s, -1), vals.repeat_interleave(g, 1)).reshape(-1)
        assert torch.allclose(out[b].float(), ref, atol=2e-2, rtol=2e-2), (b, (out[b].float() - ref).abs().max())
        lse = torch.logsumexp(s, -1)
        got = eml[b, :, 0] + torch.log(eml[b, :, 1])
        assert torch.allclose(got, lse, atol=1e-2)


def test_route_topk_exact_with_ties(ext):
    torch.manual_seed(2)
    B, C, D, k = 4, 1000, 64, 16
    gists = F.normalize(torch.randn(C + 8, D, device="cuda"), dim=-1)
    gists[10] = gists[3]  # exact tie: lower id must win
    query = torch.randn(B, D, device="cuda")
    query[0] = gists[3] * 2
    approx = (F.normalize(query, dim=-1).bfloat16().float() @ gists.bfloat16().float().t()).contiguous()
    start = torch.tensor([0, 0, 100, 990], device="cuda", dtype=torch.int32)
    end = torch.tensor([C, 500, 900, C], device="cuda", dtype=torch.int32)
    clen = torch.full((C + 8,), 8, device="cuda", dtype=torch.int32)
    clen[::7] = 5
    row0 = torch.arange(C + 8, device="cuda", dtype=torch.int32) * 8
    mem_idx, mem_len, sel = ext.route_topk(approx, query, gists, start, end, clen, row0, k, 64, -1, k * 8, False, 0, 1, 1)
    exact = F.normalize(query, dim=-1) @ gists.t()
    for b in range(B):
        ids = list(range(int(start[b]), int(end[b])))
        order = sorted(ids, key=lambda c: (-float(exact[b, c]), c))[:k]
        want = sorted(order)
        got = [int(c) for c in sel[b] if int(c) >= 0]
        assert got == want, (b, got, want)
        rows = [int(row0[c]) + t for c in want for t in range(int(clen[c]))]
        assert int(mem_len[b]) == len(rows)
        assert mem_idx[b, : len(rows)].tolist() == rows
    assert 3 in [int(c) for c in sel[0]] and 10 in [int(c) for c in sel[0]]
    # a token budget keeps whole chunks greedily in score order
    mem_idx, mem_len, sel = ext.route_topk(approx, query, gists, start, end, clen, row0, k, 64, 20, k * 8, False, 0, 1, 1)
    assert int(mem_len.max()) <= 20


def _tiny_setup(seed=0):
    from pdattention_b200.models.llama import PRALlamaReference, tiny_llama

    torch.manual_seed(seed)
    cfg = tiny_llama(head_dim=64, hidden_size=128, num_attention_heads=4, num_key_value_heads=2, chunk_tokens=16,
                     top_k_chunks=3)
    model = PRALlamaReference(cfg).eval()
    model.reset_parameters(seed=seed, std=0.08)
    C = 12
    chunks = torch.randint(0, cfg.vocab_size, (C, 16))
    lengths = torch.tensor([16, 16, 11, 16, 16, 9, 16, 16, 16, 13, 16, 16])
    return cfg, model, chunks, lengths


def test_engine_memory_build_matches_oracle(ext):
    from pdattention_b200.inference.llama_engine import LlamaWeights, PRALlamaEngine

    cfg, model, chunks, lengths = _tiny_setup()
    ref = model.encode_chunks(chunks, lengths)
    engine = PRALlamaEngine(LlamaWeights.from_reference(model, "cuda"), "cuda")
    mem = engine.build_memory(chunks, lengths, batch_chunks=5)
    for li in range(cfg.num_hidden_layers):
        for c in range(chunks.shape[0]):
            n = int(lengths[c])
            k = mem.k(li)[c * 16: c * 16 + n].float().cpu()
            assert torch.allclose(k, ref.k[li][c, :n].reshape(n, -1), atol=5e-2, rtol=5e-2), (li, c)
            v = mem.v(li)[c * 16: c * 16 + n].float().cpu()
            assert torch.allclose(v, ref.v[li][c, :n].reshape(n, -1), atol=5e-2, rtol=5e-2), (li, c)
        gref = F.normalize(ref.gist[li], dim=-1)
        assert torch.allclose(mem.gn[li][: chunks.shape[0], 0].cpu(), gref, atol=2e-2)


def test_engine_prefill_and_decode_match_oracle(ext):
    from pdattention_b200.inference.llama_engine import LlamaWeights, PRALlamaEngine
    from pdattention_b200.models.llama import reference_step

    cfg, model, chunks, lengths = _tiny_setup(1)
    ref_mem = model.encode_chunks(chunks, lengths)
    engine = PRALlamaEngine(LlamaWeights.from_reference(model, "cuda"), "cuda", decode_split_keys=64)
    engine.build_memory(chunks, lengths)
    spans = [(0, 12), (0, 6), (4, 12)]
    engine.set_namespace(torch.tensor([s for s, _ in spans]), torch.tensor([e for _, e in spans]))
    B, T = 3, 20
    plen = torch.tensor([20, 13, 7])
    ids = torch.randint(0, cfg.vocab_size, (B, T))
    logits = engine.prefill(ids, plen, max_new_tokens=4).float().cpu()
    sel0 = {li: s.cpu() for li, s in engine.last_selection.items()}
    caches = [[[None, None] for _ in range(cfg.num_hidden_layers)] for _ in range(B)]
    agree = total = 0
    for b in range(B):
        ns = list(range(*spans[b]))
        ref_logits, picks = reference_step(model, ids[b, : int(plen[b])], caches[b], ref_mem, ns)
        ref = ref_logits[-1]
        cos = F.cosine_similarity(logits[b], ref, dim=0)
        assert cos > 0.995, (b, float(cos))
        for li, p in enumerate(picks):
            got = [int(c) for c in sel0[li][b] if int(c) >= 0]
            agree += len(set(got) & set(p))
            total += len(p)
        assert [int(c) for c in sel0[0][b] if int(c) >= 0] == picks[0]
    assert agree >= 0.9 * total
    # teacher-forced decode steps
    for step in range(3):
        tok = torch.randint(0, cfg.vocab_size, (B,))
        got = engine.decode_step(tok).float().cpu()
        for b in range(B):
            ref_logits, _ = reference_step(model, tok[b: b + 1], caches[b], ref_mem, list(range(*spans[b])))
            cos = F.cosine_similarity(got[b], ref_logits[-1], dim=0)
            assert cos > 0.99, (step, b, float(cos))


def test_long_prompt_implicit_head_matches_oracle(ext):
    from pdattention_b200.inference.llama_engine import LlamaWeights, PRALlamaEngine
    from pdattention_b200.inference.long_prompt import long_prompt_generate
    from pdattention_b200.models.llama import reference_step

    cfg, model, _, _ = _tiny_setup(2)
    gen = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=gen).tolist() for n in (70, 40, 20)]
    engine = PRALlamaEngine(LlamaWeights.from_reference(model, "cuda"), "cuda", decode_split_keys=64)
    tokens, plan, first = long_prompt_generate(engine, prompts, 3, direct_window=16)
    assert tokens.shape == (3, 3)
    assert plan.position_offset.tolist() == [54, 24, 4]
    mem = model.encode_chunks(plan.chunks, plan.chunk_lengths)
    for b in range(3):
        cache = [[None, None] for _ in range(cfg.num_hidden_layers)]
        ns = list(range(int(plan.ns_start[b]), int(plan.ns_end[b])))
        tail = plan.tails[b, : int(plan.tail_lengths[b])]
        ref, _ = reference_step(model, tail, cache, mem, ns, position_offset=int(plan.position_offset[b]))
        cos = F.cosine_similarity(first[b].float().cpu(), ref[-1], dim=0)
        assert cos > 0.995, (b, float(cos))


def test_graphed_decode_matches_eager(ext):
    from pdattention_b200.inference.llama_engine import LlamaWeights, PRALlamaEngine

    cfg, model, chunks, lengths = _tiny_setup(4)
    weights = LlamaWeights.from_reference(model, "cuda")
    outs = []
    for graphed in (False, True):
        engine = PRALlamaEngine(weights, "cuda", decode_split_keys=64)
        engine.build_memory(chunks, lengths)
        engine.set_namespace(torch.zeros(2, dtype=torch.int32), torch.full((2,), 12, dtype=torch.int32))
        tok = engine.prefill(torch.arange(24).view(2, 12) % cfg.vocab_size, torch.tensor([12, 9]), 6).float().argmax(-1)
        tok = engine.decode_step(tok).float().argmax(-1)
        step = engine.decode_step
        if graphed:
            engine.capture_decode()
            step = engine.decode_step_graphed
        seq = []
        for _ in range(4):
            logits = step(tok).float().clone()
            seq.append(logits)
            tok = logits.argmax(-1)
        outs.append(torch.stack(seq))
        assert engine.cache_len.tolist() == [12 + 5, 9 + 5]
    assert torch.allclose(outs[0], outs[1], atol=1e-3), (outs[0] - outs[1]).abs().max()


def test_sharded_routing_merge_equals_unsharded(ext):
    """Local top-k per chunk slice + merge of the slices' candidates == routing over all chunks."""
    torch.manual_seed(5)
    B, C, D, k = 6, 800, 128, 16
    gists = F.normalize(torch.randn(C, D, device="cuda"), dim=-1)
    query = torch.randn(B, D, device="cuda")
    scores = (F.normalize(query, dim=-1).bfloat16().float() @ gists.bfloat16().float().t()).contiguous()
    start = torch.tensor([0, 0, 50, 300, 0, 790], device="cuda", dtype=torch.int32)
    end = torch.tensor([C, 200, 700, 420, C, C], device="cuda", dtype=torch.int32)
    clen = torch.full((C,), 64, device="cuda", dtype=torch.int32)
    row0 = torch.arange(C, device="cuda", dtype=torch.int32) * 64
    want = ext.route_topk(scores, query, gists, start, end, clen, row0, k, 64, 640, k * 64, False, 0, 1, 1)
    world, per = 4, C // 4
    blocks = []
    for r in range(world):
        c0, c1 = r * per, (r + 1) * per
        lo = (start - c0).clamp(0, per).to(torch.int32)
        hi = (end - c0).clamp(0, per).to(torch.int32)
        cs, ci = ext.route_topk(scores[:, c0:c1].contiguous(), query, gists[c0:c1].contiguous(), lo, hi, clen, row0, k,
                                64, -1, 0, True, c0, 1, 1)
        blocks.append(torch.cat([cs, ci.view(torch.float32)], dim=1))
    got = ext.route_merge(torch.cat(blocks, dim=1).contiguous(), world, k, 640, clen, row0, k * 64, False)
    assert torch.equal(got[1], want[1])
    assert torch.equal(got[2], want[2])
    for b in range(B):
        n = int(want[1][b])
        assert torch.equal(got[0][b, :n], want[0][b, :n])


def test_memory_sweep_fused_step_matches_torch_baseline(ext):
    from pdattention_b200.inference.memory_sweep import (HEAD_DIM, HEADS, KV_DIM, ShardedLayerMemory,
                                                         baseline_layer_step, fused_layer_step)

    mem = ShardedLayerMemory(1 << 16, 4, "cuda", seed=1)
    gen = torch.Generator(device="cuda").manual_seed(3)
    rq = torch.randn((8, KV_DIM), generator=gen, device="cuda")
    q = torch.randn((8, HEADS * HEAD_DIM), generator=gen, device="cuda").bfloat16()
    for k in (4, 16):
        got = fused_layer_step(mem, rq, q, k).float()
        want = baseline_layer_step(mem, rq, q, k).float()
        assert torch.allclose(got, want, atol=3e-2, rtol=3e-2), (k, (got - want).abs().max())


def test_segmented_selection_equals_single_pass(ext, monkeypatch):
    """Rows cut into segments (one CTA each) + on-GPU merge == one CTA per row."""
    from pdattention_b200.inference import routing

    torch.manual_seed(6)
    B, C, D, k = 5, 3000, 64, 8
    for G in (1, 4):
        gists = F.normalize(torch.randn(C * G, D, device="cuda"), dim=-1)
        query = torch.randn(B, D, device="cuda")
        scores = (F.normalize(query, dim=-1).bfloat16().float() @ gists.bfloat16().float().t()).contiguous()
        start = torch.tensor([0, 100, 0, 2500, 7], device="cuda", dtype=torch.int32)
        end = torch.tensor([C, 2900, 1000, C, 8], device="cuda", dtype=torch.int32)
        clen = torch.full((C,), 16, device="cuda", dtype=torch.int32)
        row0 = torch.arange(C, device="cuda", dtype=torch.int32) * 16
        want = ext.route_topk(scores, query, gists, start, end, clen, row0, k, 32, 100, k * 16, False, 0, G, 1)
        monkeypatch.setattr(routing, "SEGMENT", 256)
        got = routing.select_chunks(ext, scores, query, gists, start, end, clen, row0, k, 32, 100, k * 16,
                                    gists_per_chunk=G)
        monkeypatch.setattr(routing, "SEGMENT", 8192)
        assert torch.equal(got[1], want[1]) and torch.equal(got[2], want[2]), (G, got[2], want[2])


def test_host_resident_chunk_memory_equals_device_memory(ext):
    """kv_residency="cpu": the chunk K/V pool moves to pinned host memory after the build and the
    prefill / decode attention gathers the selected rows over the host link: same logits."""
    from pdattention_b200.inference.llama_engine import LlamaWeights, PRALlamaEngine

    cfg, model, chunks, lengths = _tiny_setup(2)
    weights = LlamaWeights.from_reference(model, "cuda")
    out = {}
    for residency in ("gpu", "cpu"):
        engine = PRALlamaEngine(weights, "cuda", decode_split_keys=64, kv_residency=residency)
        mem = engine.build_memory(chunks, lengths)
        assert mem.pool.is_cuda == (residency == "gpu")
        engine.set_namespace(torch.tensor([0, 0]), torch.tensor([12, 6]))
        ids = torch.randint(0, cfg.vocab_size, (2, 9), generator=torch.Generator().manual_seed(3))
        first = engine.prefill(ids, torch.tensor([9, 5]), max_new_tokens=3).float().cpu()
        step = engine.decode_step(first.argmax(-1).cuda()).float().cpu()
        out[residency] = (first, step)
    assert torch.equal(out["gpu"][0], out["cpu"][0])
    assert torch.equal(out["gpu"][1], out["cpu"][1])


@pytest.mark.parametrize("head_dim,run,mem_len", [(128, 64, 1024), (128, 40, 600), (64, 64, 100), (128, 64, 0)])
def test_tma_decode_attention_matches_cp_async_kernel(ext, head_dim, run, mem_len):
    """The TMA-fed decode kernel (selected chunks as 64-row runs of the pool -> one box per 64
    columns; other runs gathered into the same swizzled layout) equals the cp.async kernel and
    the fp32 softmax."""
    torch.manual_seed(8)
    B, H, Hkv, max_len, tc = 5, 16, 4, 700, 64
    chunks = 40
    q = torch.randn(B, H * head_dim, device="cuda").bfloat16()
    pool = torch.randn(chunks * tc, 2 * Hkv * head_dim, device="cuda").bfloat16()
    mk, mv = pool[:, : Hkv * head_dim], pool[:, Hkv * head_dim:]
    mem_idx = torch.zeros(B, max(mem_len, 1), device="cuda", dtype=torch.int32)
    for b in range(B):  # runs of `run` consecutive rows from distinct chunks
        picks = torch.randperm(chunks)[: (mem_len + run - 1) // run + 1]
        rows = torch.cat([c * tc + torch.arange(run) for c in picks.tolist()])[:mem_len]
        mem_idx[b, :mem_len] = rows.to(torch.int32).cuda()
    lens = torch.tensor([mem_len, mem_len // 2, mem_len, 0, mem_len], device="cuda", dtype=torch.int32)
    cache = torch.randn(2, B, max_len, Hkv * head_dim, device="cuda").bfloat16()
    loc_len = torch.tensor([700, 1, 333, 64, 129], device="cuda", dtype=torch.int32)
    args = (mk, mv, mem_idx, lens, cache[0], cache[1], loc_len, mem_len + max_len, 512, True)
    try:
        ext.decode_set_tma(True)
        out_t, eo_t, eml_t = ext.decode_attention(q, H, Hkv, head_dim, *args)
        ext.decode_set_tma(False)
        out_c, eo_c, eml_c = ext.decode_attention(q, H, Hkv, head_dim, *args)
    finally:
        ext.decode_set_tma(True)
    assert torch.allclose(out_t.float(), out_c.float(), atol=1e-2, rtol=1e-2), (out_t.float() - out_c.float()).abs().max()
    assert torch.allclose(eml_t, eml_c, atol=1e-3, rtol=1e-3)
    g = H // Hkv
    for b in range(B):
        n_m, n_l = int(lens[b]), int(loc_len[b])
        keys = torch.cat([mk[mem_idx[b, :n_m].long()], cache[0, b, :n_l]]).float().view(-1, Hkv, head_dim)
        vals = torch.cat([mv[mem_idx[b, :n_m].long()], cache[1, b, :n_l]]).float().view(-1, Hkv, head_dim)
        s = torch.einsum("hd,khd->hk", q[b].float().view(H, head_dim), keys.repeat_interleave(g, 1)) / math.sqrt(head_dim)
        ref = torch.einsum("hk,khd->hd", torch.softmax(s, -1), vals.repeat_interleave(g, 1)).reshape(-1)
        assert torch.allclose(out_t[b].float(), ref, atol=2e-2, rtol=2e-2), (b, (out_t[b].float() - ref).abs().max())


@pytest.mark.parametrize("tma", [True, False])
def test_phase_split_decode_attention_equals_single_launch(ext, tma):
    """Memory splits, local splits (launched first, on another stream, before the memory row
    lists exist) and a separate merge give the single launch's output."""
    torch.manual_seed(11)
    B, H, Hkv, D, max_len, tc, chunks, sk = 4, 16, 4, 128, 600, 64, 30, 256
    q = torch.randn(B, H * D, device="cuda").bfloat16()
    pool = torch.randn(chunks * tc, 2 * Hkv * D, device="cuda").bfloat16()
    mk, mv = pool[:, : Hkv * D], pool[:, Hkv * D:]
    mem_max = 8 * tc
    mem_idx = torch.zeros(B, mem_max, device="cuda", dtype=torch.int32)
    for b in range(B):
        picks = torch.randperm(chunks)[:8]
        mem_idx[b] = torch.cat([c * tc + torch.arange(tc) for c in picks.tolist()]).to(torch.int32).cuda()
    mem_len = torch.tensor([mem_max, 100, 0, 448], device="cuda", dtype=torch.int32)
    cache = torch.randn(2, B, max_len, Hkv * D, device="cuda").bfloat16()
    loc_len = torch.tensor([600, 1, 257, 64], device="cuda", dtype=torch.int32)
    try:
        ext.decode_set_tma(tma)
        ref = ext.decode_attention(q, H, Hkv, D, mk, mv, mem_idx, mem_len, cache[0], cache[1], loc_len,
                                   mem_max + max_len, sk, False)[0]
        msk = 128  # finer memory splits than local ones
        n_mem, n_loc = mem_max // msk, -(-max_len // sk)
        part_o = torch.full((B, H, n_mem + n_loc, D), float("nan"), device="cuda")
        part_ml = torch.full((B, H, n_mem + n_loc, 2), float("nan"), device="cuda")
        common = dict(mem_splits=n_mem, mem_split_keys=msk, part_o=part_o, part_ml=part_ml)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):  # a persistent grid of 7 CTAs walks the local splits
            ext.decode_attention(q, H, Hkv, D, None, None, None, None, cache[0], cache[1], loc_len, 0, sk, False,
                                 split_lo=n_mem, split_count=n_loc, phase=1, max_ctas=7, **common)
        ext.decode_attention(q, H, Hkv, D, mk, mv, mem_idx, mem_len, cache[0], cache[1], loc_len, 0, sk, False,
                             split_lo=0, split_count=n_mem, phase=1, **common)
        torch.cuda.current_stream().wait_stream(side)
        out = ext.decode_attention(q, H, Hkv, D, None, None, None, None, cache[0], cache[1], loc_len, 0, sk, False,
                                   phase=2, **common)[0]
    finally:
        ext.decode_set_tma(True)
    assert not torch.isnan(part_ml).any()
    assert torch.allclose(out.float(), ref.float(), atol=1e-2, rtol=1e-2), (out.float() - ref.float()).abs().max()


@pytest.mark.parametrize("graphed", [False, True])
def test_overlapped_routing_decode_equals_serial(ext, graphed):
    """Decode with routing on the side stream (local splits concurrent) matches the serial step
    up to the summation order of the split layout, and repeats bit for bit (no race between the
    streams)."""
    from pdattention_b200.inference.llama_engine import LlamaWeights, PRALlamaEngine

    cfg, model, chunks, lengths = _tiny_setup(5)
    weights = LlamaWeights.from_reference(model, "cuda")
    feed = torch.randint(0, cfg.vocab_size, (4, 2), generator=torch.Generator().manual_seed(9)).cuda()
    outs = []
    for overlap in (False, True, True):
        engine = PRALlamaEngine(weights, "cuda", decode_split_keys=64, overlap_routing=overlap)
        engine.build_memory(chunks, lengths)
        engine.set_namespace(torch.tensor([0, 3], dtype=torch.int32), torch.tensor([12, 9], dtype=torch.int32))
        engine.prefill(torch.arange(24).view(2, 12) % cfg.vocab_size, torch.tensor([12, 9]), 6)
        engine.decode_step(feed[0])
        step = engine.decode_step
        if graphed:
            engine.capture_decode()
            step = engine.decode_step_graphed
        outs.append(torch.stack([step(feed[i]).float().clone() for i in range(1, 4)]))
    assert torch.equal(outs[1], outs[2])
    cos = F.cosine_similarity(outs[0].flatten(0, 1), outs[1].flatten(0, 1), dim=-1)
    assert cos.min() > 0.9999, cos
    assert (outs[0] - outs[1]).abs().max() < 0.1
