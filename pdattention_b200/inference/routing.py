"""Exact top-k chunk routing on the device, from one GPU to a chunk-sharded group.

Scores come from a tensor-core GEMM (bf16 normalised queries x bf16 normalised gists);
``select_chunks`` turns them into the exact fp32 top-k per row:

* a row's chunks are cut into segments of up to ``SEGMENT`` chunks, one CTA each, so a
  large memory (a 16M-token memory has 262,144 chunks) spreads over the whole GPU; each
  segment radix-selects its candidates and rescores them in fp32;
* the segments' candidates are merged on the GPU (``route_merge``);
* across GPUs (chunk-sharded memory) each rank's merged top-k candidates are
  exchanged over NVLink peer stores and merged again, identically on every rank; with
  one segment per row (up to 8,192 chunks per rank) the exchange and the merge are fused
  into the routing kernel itself (``TensorParallel.route_exchange``).

Ties break towards the lower chunk id; the greedy token budget and the memory row list
(only rows this rank holds) are produced by the final merge.
"""

from __future__ import annotations

import math

import torch

SEGMENT = 8192
MAX_CANDIDATES = 512


def segments_for(n_chunks: int, k: int) -> int:
    want = max(1, math.ceil(n_chunks / SEGMENT))
    return max(1, min(want, MAX_CANDIDATES // max(k, 1)))


def select_chunks(ext, scores, query, gists, start, end, chunk_len, chunk_row0, k: int, k_cand: int, budget: int,
                  mem_max: int, *, gists_per_chunk: int = 1, id_offset: int = 0, comm=None,
                  global_len=None, global_row0=None, pool_rows: int = -1, page_table=None):
    """``(mem_idx, mem_len, selected ids)`` for every row.  ``scores`` ``[B, C_local * G]``;
    with ``comm`` the chunk ids are global (``id_offset`` = this rank's first chunk) and
    ``global_len`` / ``global_row0`` describe every chunk (row0 < 0: held by another rank).
    ``pool_rows`` (the memory pool's row count) lets the bounds-checked kernels verify the row
    lists they write.  ``page_table`` ``[B, P]`` (a paged chunk cache) maps each row's namespace
    positions to chunk ids; it needs one segment per row."""
    G = gists_per_chunk
    n = scores.shape[1] // G
    S = segments_for(n, k)
    world = comm.world if comm is not None else 1
    if page_table is not None:
        if world != 1 or page_table.shape[1] > SEGMENT:
            raise ValueError("a page table needs unsharded routing and at most 8,192 pages per row")
        return ext.route_topk(scores, query, gists, start, end, chunk_len, chunk_row0, k, k_cand, budget, mem_max,
                              False, 0, G, 1, pool_rows, page_table)
    if world == 1 and S == 1:
        return ext.route_topk(scores, query, gists, start, end, chunk_len, chunk_row0, k, k_cand, budget, mem_max,
                              False, 0, G, 1, pool_rows)
    rows = query.shape[0]
    if world > 1 and S == 1 and hasattr(comm, "route_exchange") and rows <= comm.decode_rows and \
            k <= comm.ROUTE_K_MAX and world * k <= MAX_CANDIDATES:
        return comm.route_exchange(scores, query, gists, start, end, k, k_cand, budget, mem_max, id_offset, G,
                                   global_len, global_row0, pool_rows)
    cs, ci = ext.route_topk(scores, query, gists, start, end, chunk_len, chunk_row0, k, k_cand, -1, 0, True,
                            id_offset, G, S)
    if S > 1:
        blocks = torch.cat([cs.view(rows, S, k), ci.view(torch.float32).view(rows, S, k)], dim=2).view(rows, -1)
        if world == 1:
            return ext.route_merge(blocks, S, k, budget, chunk_len, chunk_row0, mem_max, False, pool_rows)
        cs, ci = ext.route_merge(blocks, S, k, -1, chunk_len, chunk_row0, 0, True)
    merged = comm.all_gather_columns(torch.cat([cs, ci.view(torch.float32)], dim=1))
    return ext.route_merge(merged, world, k, budget, global_len, global_row0, mem_max, False, pool_rows)
