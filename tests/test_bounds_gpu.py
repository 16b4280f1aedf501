"""Bounds-checked variants of the gather (decode attention) and routing kernels.

With ``set_bounds_check(True)`` a kernel that meets an out-of-range index records
it in the device's status word and skips that access; the test feeds such
indices and checks both the record and that the output equals the fp32
PyTorch restatement over the in-range keys only.  On in-range inputs the
checked and unchecked variants agree exactly and the status stays clean.
The unchecked variants never see a bad index here.
"""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DECODE_MEM_ROW, ROUTE_NAMESPACE, ROUTE_POOL_ROW = 3, 4, 5


@pytest.fixture
def ext():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from pdattention_b200.ops import _ext

    module = _ext.require()
    module.set_bounds_check(True)
    module.bounds_reset(0)
    yield module
    module.bounds_reset(0)
    module.set_bounds_check(False)


def _reference(q, mk, mv, cache, idx_rows, n_loc, H, Hkv, dh):
    g = H // Hkv
    keys = torch.cat([mk[idx_rows], cache[0, :n_loc]]).float().view(-1, Hkv, dh).repeat_interleave(g, 1)
    vals = torch.cat([mv[idx_rows], cache[1, :n_loc]]).float().view(-1, Hkv, dh).repeat_interleave(g, 1)
    s = torch.einsum("hd,khd->hk", q.float().view(H, dh), keys) / math.sqrt(dh)
    return torch.einsum("hk,khd->hd", torch.softmax(s, -1), vals).reshape(-1)


def test_decode_skips_and_records_a_row_outside_the_pool(ext):
    torch.manual_seed(3)
    B, H, Hkv, dh, rows, max_len = 2, 8, 2, 128, 400, 96
    q = torch.randn(B, H * dh, device="cuda").bfloat16()
    pool = torch.randn(rows, 2 * Hkv * dh, device="cuda").bfloat16()
    mk, mv = pool[:, : Hkv * dh], pool[:, Hkv * dh:]
    mem_idx = torch.randint(0, rows, (B, 80), device="cuda", dtype=torch.int32)
    mem_len = torch.tensor([80, 50], device="cuda", dtype=torch.int32)
    cache = torch.randn(2, B, max_len, Hkv * dh, device="cuda").bfloat16()
    loc_len = torch.tensor([40, 96], device="cuda", dtype=torch.int32)
    args = (mk, mv, mem_idx, mem_len, cache[0], cache[1], loc_len, 80 + max_len, 64, False)
    clean = ext.decode_attention(q, H, Hkv, dh, *args)[0].clone()
    assert ext.bounds_status(0) == [0, 0, 0, 0]
    ext.set_bounds_check(False)
    unchecked = ext.decode_attention(q, H, Hkv, dh, *args)[0]
    ext.set_bounds_check(True)
    assert torch.equal(clean, unchecked)

    bad = mem_idx.clone()
    bad[0, 17] = rows + 7  # one key of row 0 points past the pool
    out = ext.decode_attention(q, H, Hkv, dh, mk, mv, bad, *args[3:])[0]
    torch.cuda.synchronize()
    code, kernel, index, limit = ext.bounds_status(0)
    assert (code, kernel, index, limit) == (1, DECODE_MEM_ROW, rows + 7, rows)
    keep = [j for j in range(80) if j != 17]
    ref0 = _reference(q[0], mk, mv, cache[:, 0], mem_idx[0, keep].long(), 40, H, Hkv, dh)
    assert torch.allclose(out[0].float(), ref0, atol=2e-2, rtol=2e-2)
    assert torch.equal(out[1], clean[1])  # the other row is untouched


def test_routing_clamps_a_namespace_outside_the_chunk_table(ext):
    torch.manual_seed(4)
    B, C, D, k, tc = 3, 200, 64, 4, 16
    gists = torch.nn.functional.normalize(torch.randn(C, D, device="cuda"), dim=-1)
    query = torch.randn(B, D, device="cuda")
    scores = (torch.nn.functional.normalize(query, dim=-1) @ gists.t()).contiguous()
    clen = torch.full((C,), tc, device="cuda", dtype=torch.int32)
    row0 = torch.arange(C, device="cuda", dtype=torch.int32) * tc
    start = torch.tensor([0, 50, 120], device="cuda", dtype=torch.int32)
    end = torch.tensor([C, 90, C], device="cuda", dtype=torch.int32)
    want = ext.route_topk(scores, query, gists, start, end, clen, row0, k, 32, -1, k * tc, False, 0, 1, 1, C * tc)
    assert ext.bounds_status(0) == [0, 0, 0, 0]
    wide = end.clone()
    wide[2] = C + 55  # row 2's namespace runs past the table
    got = ext.route_topk(scores, query, gists, start, wide, clen, row0, k, 32, -1, k * tc, False, 0, 1, 1, C * tc)
    torch.cuda.synchronize()
    assert ext.bounds_status(0)[:2] == [1, ROUTE_NAMESPACE]
    for a, b in zip(want, got):
        assert torch.equal(a, b)


def test_routing_marks_rows_past_the_pool(ext):
    torch.manual_seed(5)
    B, C, D, k, tc = 2, 64, 32, 3, 8
    gists = torch.nn.functional.normalize(torch.randn(C, D, device="cuda"), dim=-1)
    query = torch.randn(B, D, device="cuda")
    gists[C - 1] = torch.nn.functional.normalize(query[0], dim=-1)  # row 0's best chunk is the last one
    scores = (torch.nn.functional.normalize(query, dim=-1) @ gists.t()).contiguous()
    clen = torch.full((C,), tc, device="cuda", dtype=torch.int32)
    row0 = torch.arange(C, device="cuda", dtype=torch.int32) * tc
    start = torch.zeros(B, device="cuda", dtype=torch.int32)
    end = torch.full((B,), C, device="cuda", dtype=torch.int32)
    pool_rows = (C - 1) * tc + 3  # the last chunk's rows 3.. lie past this (too short) pool
    mem_idx, mem_len, sel = ext.route_topk(scores, query, gists, start, end, clen, row0, k, 16, -1, k * tc, False, 0,
                                           1, 1, pool_rows)
    torch.cuda.synchronize()
    assert int(sel[0].max()) == C - 1
    assert ext.bounds_status(0)[:2] == [1, ROUTE_POOL_ROW]
    n0 = int(mem_len[0])
    rows0 = mem_idx[0, :n0]
    assert int((rows0 == -1).sum()) == tc - 3  # the last chunk's rows past the pool are marked, not written
    assert int(rows0.max()) < pool_rows
