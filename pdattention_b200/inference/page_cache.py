"""A persistent, deduplicated chunk memory for the Llama-family engine (device page pool).

A *page* is one chunk: ``chunk_tokens`` K/V rows of every layer (this rank's KV heads under
tensor parallelism) plus its routing gist.  References are added by content: a reference's
fingerprint (sha256 of its token ids and the chunk size) names an entry that owns a
contiguous run of pages, so the same content added again -- by another request, or by
another row of the same batch -- reuses the pages (reference counted) instead of being
encoded twice.  When the pool is full, unreferenced entries are evicted least recently
used first; with a host tier their pages (K/V rows, gists, lengths) move to pinned host
memory and come back with one host-to-device copy when the content is added again.

Rows read their own references through a page table: ``page_table(rows)`` lists, per
batch row, the pages of the entries that row may see, and the engine's routing kernel
scores and selects through that indirection (``route_topk`` with ``page_table``), so one
pool serves a batch whose rows have different, overlapping reference sets.  This is the
device counterpart of the reference's cache services and row-isolated namespaces
(``src/pra_torch/cache_services.py:27-32``, ``src/pra_torch/memory.py:1217-1309``).
"""

from __future__ import annotations

import hashlib
from collections import OrderedDict
from dataclasses import dataclass, field

import numpy as np
import torch


@dataclass
class PageEntry:
    """One reference's pages: ``[first, first + pages)`` of the pool."""

    fingerprint: str
    first: int
    pages: int
    lengths: list[int]
    uris: set = field(default_factory=set)
    refs: int = 0


@dataclass
class _HostCopy:
    kv: torch.Tensor       # [L, pages * tc, 2 * kv_dim] pinned
    gists: torch.Tensor    # [3, L, pages, 1, gist_dim] pinned
    gn_bf16: torch.Tensor  # [L, pages, gist_dim] pinned
    count: torch.Tensor    # [L, pages] pinned
    lengths: list[int]


def fingerprint(token_ids, chunk_tokens: int) -> str:
    ids = np.asarray(token_ids, dtype=np.int64)
    return hashlib.sha256(ids.tobytes() + chunk_tokens.to_bytes(4, "little")).hexdigest()


class PageAllocator:
    """First-fit allocator of contiguous page runs over ``capacity`` pages (free runs merged)."""

    def __init__(self, capacity: int):
        self.capacity = capacity
        self.free: list[list[int]] = [[0, capacity]]  # sorted [start, length] runs

    def allocate(self, n: int) -> int | None:
        for run in self.free:
            if run[1] >= n:
                start = run[0]
                run[0] += n
                run[1] -= n
                if run[1] == 0:
                    self.free.remove(run)
                return start
        return None

    def release(self, start: int, n: int) -> None:
        self.free.append([start, n])
        self.free.sort()
        merged: list[list[int]] = []
        for s, length in self.free:
            if merged and merged[-1][0] + merged[-1][1] == s:
                merged[-1][1] += length
            else:
                merged.append([s, length])
        self.free = merged

    def free_pages(self) -> int:
        return sum(length for _, length in self.free)


class PagedChunkCache:
    """Device page pool of encoded reference chunks for one ``PRALlamaEngine`` (or TP shard).

    ``add(token_ids, uri)`` returns the reference's ``PageEntry`` (encoding it only when its
    content is new), ``release(entry)`` drops one holder, ``page_table(rows)`` builds the
    routing indirection of a batch and installs it on the engine.  ``host_capacity_pages``
    (0: none) sizes the pinned host tier that evicted entries move to.
    """

    def __init__(self, engine, capacity_pages: int, chunk_tokens: int | None = None, host_capacity_pages: int = 0,
                 batch_chunks: int = 256):
        from .llama_engine import ChunkMemory

        cfg = engine.cfg
        self.engine = engine
        self.tc = chunk_tokens or cfg.chunk_tokens
        self.memory = ChunkMemory(cfg, capacity_pages, engine.kv_dim, engine.device, self.tc, gist_dim=cfg.kv_dim)
        self.allocator = PageAllocator(capacity_pages)
        self.entries: dict[str, PageEntry] = {}
        self.by_uri: dict[str, PageEntry] = {}
        self.lru: OrderedDict[str, None] = OrderedDict()  # unreferenced entries, oldest first
        self.host: OrderedDict[str, _HostCopy] = OrderedDict()
        self.host_capacity = host_capacity_pages
        self.batch_chunks = batch_chunks
        self.stats = {"encoded_pages": 0, "reused_entries": 0, "evicted_entries": 0, "restored_entries": 0,
                      "host_dropped_entries": 0}
        engine.memory = self.memory

    # -- entries -------------------------------------------------------------------
    def _chunks(self, token_ids) -> tuple[torch.Tensor, list[int]]:
        ids = [int(t) for t in token_ids]
        n = max(1, -(-len(ids) // self.tc))
        out = torch.zeros((n, self.tc), dtype=torch.long)
        lengths = []
        for i in range(n):
            piece = ids[i * self.tc:(i + 1) * self.tc]
            out[i, : len(piece)] = torch.tensor(piece, dtype=torch.long)
            lengths.append(len(piece))
        return out, lengths

    def add(self, token_ids, uri: str | None = None) -> PageEntry:
        fp = fingerprint(token_ids, self.tc)
        entry = self.entries.get(fp)
        if entry is not None:
            self.stats["reused_entries"] += 1
        else:
            chunks, lengths = self._chunks(token_ids)
            first = self._allocate(len(lengths))
            copy = self.host.pop(fp, None)
            if copy is not None:
                self._restore(copy, first)
                self.stats["restored_entries"] += 1
            else:
                self.engine.encode_into(self.memory, chunks, torch.tensor(lengths, dtype=torch.int32), first,
                                        self.batch_chunks)
                self.stats["encoded_pages"] += len(lengths)
            entry = PageEntry(fp, first, len(lengths), lengths)
            self.entries[fp] = entry
        if entry.refs == 0:
            self.lru.pop(fp, None)
        entry.refs += 1
        if uri is not None:
            entry.uris.add(uri)
            self.by_uri[uri] = entry
        return entry

    def release(self, entry: PageEntry | str) -> None:
        if isinstance(entry, str):
            entry = self.by_uri[entry]
        if entry.refs <= 0:
            raise ValueError("release of an entry nobody holds")
        entry.refs -= 1
        if entry.refs == 0:
            self.lru[entry.fingerprint] = None  # evictable, most recent last

    def _allocate(self, n: int) -> int:
        if n > self.allocator.capacity:
            raise ValueError(f"a reference of {n} pages exceeds the pool ({self.allocator.capacity} pages)")
        while True:
            first = self.allocator.allocate(n)
            if first is not None:
                return first
            if not self.lru:
                raise RuntimeError("page pool full: every entry is referenced (release entries or grow the pool)")
            self._evict(next(iter(self.lru)))

    def _evict(self, fp: str) -> None:
        entry = self.entries.pop(fp)
        self.lru.pop(fp, None)
        for uri in entry.uris:
            if self.by_uri.get(uri) is entry:
                del self.by_uri[uri]
        if self.host_capacity > 0 and entry.pages <= self.host_capacity:
            self.host[fp] = self._to_host(entry)
            while sum(c.gn_bf16.shape[1] for c in self.host.values()) > self.host_capacity:
                self.host.popitem(last=False)
                self.stats["host_dropped_entries"] += 1
        mem = self.memory
        mem.chunk_len[entry.first: entry.first + entry.pages].zero_()
        self.allocator.release(entry.first, entry.pages)
        self.stats["evicted_entries"] += 1

    def _to_host(self, entry: PageEntry) -> _HostCopy:
        mem, s, n = self.memory, entry.first, entry.pages
        rows = slice(s * self.tc, (s + n) * self.tc)

        on_gpu = self.memory.pool.is_cuda

        def pinned(t):
            out = torch.empty(t.shape, dtype=t.dtype, pin_memory=on_gpu)
            out.copy_(t, non_blocking=on_gpu)
            return out

        copy = _HostCopy(pinned(mem.pool[:, rows]), pinned(mem.tables[:, :, s: s + n]),
                         pinned(mem.gn_bf16[:, s: s + n]), pinned(mem.count[:, s: s + n]), list(entry.lengths))
        if on_gpu:
            torch.cuda.current_stream(self.memory.pool.device).synchronize()  # the pages are reused right after
        return copy

    def _restore(self, copy: _HostCopy, first: int) -> None:
        mem, n = self.memory, len(copy.lengths)
        mem.pool[:, first * self.tc:(first + n) * self.tc].copy_(copy.kv, non_blocking=True)
        mem.tables[:, :, first: first + n].copy_(copy.gists, non_blocking=True)
        mem.gn_bf16[:, first: first + n].copy_(copy.gn_bf16, non_blocking=True)
        mem.count[:, first: first + n].copy_(copy.count, non_blocking=True)
        mem.chunk_len[first: first + n].copy_(torch.tensor(copy.lengths, dtype=torch.int32), non_blocking=True)

    # -- batches -------------------------------------------------------------------
    def page_table(self, rows: list[list[PageEntry]], install: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
        """``(table [B, P] int32, counts [B])`` on the device: row b may read the pages of its
        entries (in the order given); installed as the engine's namespace when ``install``."""
        width = max([sum(e.pages for e in row) for row in rows] + [1])
        table = np.zeros((len(rows), width), dtype=np.int32)
        counts = np.zeros(len(rows), dtype=np.int32)
        for b, row in enumerate(rows):
            pages = [p for e in row for p in range(e.first, e.first + e.pages)]
            table[b, : len(pages)] = pages
            counts[b] = len(pages)
        dev = self.engine.device
        table_t = torch.from_numpy(table).to(dev)
        counts_t = torch.from_numpy(counts).to(dev)
        if install:
            self.engine.set_page_table(table_t, counts_t)
        return table_t, counts_t

    def resident_pages(self) -> int:
        return self.allocator.capacity - self.allocator.free_pages()
