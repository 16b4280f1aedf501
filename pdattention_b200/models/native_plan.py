"""Python view of the native cache-build planner (``pra_ops.plan_batch``, ``csrc/planner.cpp``).

The C++ planner returns flat arrays (entries, chunks, per-row audit tuples) and
one packed int32 table array for the device.  This module wraps them in the
interface the device runtime already uses for a Python-made ``BatchPlan``:
``entries`` / ``chunks`` are sequences whose records are built on first access
(the training step itself never touches them), each row gets a cache object
whose resolution audit is materialised when read, and the metadata a record
carries (resolver identity fingerprints, chunk provenance) is taken from the
Python planner for that row the first time anyone asks for it.
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np

from ..chunking import chunk_identity
from ..memory.cache import PRASimpleMemoryCache
from ..memory.resolution import ResolutionEvent

_CYCLE = {"skip": 0, "error": 1, "link_only": 2}
_MISSING = {"skip": 0, "warn": 1, "error": 2}
_OVERFLOW = {"truncate": 0, "merge_tail": 1, "error": 2}


def native_config(cfg, resolver_config) -> dict | None:
    """The planner's settings for ``cfg``, or ``None`` when the native planner does not apply."""
    routing = cfg.routing_chunking_config
    if routing.mode != "fixed" or cfg.reference_encoding_strategy != "independent":
        return None
    if resolver_config is not None and (resolver_config.type != "in_memory" or resolver_config.options):
        return None  # resolver options change resolution: the Python planner handles them
    limit = int(cfg.effective_model_max_context_tokens)
    size = int(routing.chunk_tokens or limit)
    overlap = int(routing.resolved_overlap_tokens(size))
    cap = cfg.max_materialized_memory_tokens
    max_chunks = cfg.max_gists_per_reference
    return {
        "recursive": bool(cfg.recursive_refs_enabled), "max_depth": int(cfg.recursive_max_depth),
        "max_children": int(cfg.recursive_max_children_per_reference),
        "max_refs": int(cfg.recursive_max_total_references), "max_tokens": int(cfg.recursive_max_total_tokens),
        "cycle_policy": _CYCLE[cfg.recursive_cycle_policy], "missing_policy": _MISSING[cfg.recursive_missing_ref_policy],
        "limit": limit, "budget_limit": limit - int(cfg.context_safety_reserve_tokens),
        "cap": -1 if cap is None else int(cap), "chunk_size": size, "overlap": overlap,
        "max_chunks": -1 if max_chunks is None else int(max_chunks),
        "overflow": _OVERFLOW[cfg.gist_overflow_policy], "kmeans": cfg.gist_mode == "kmeans",
    }


class _Lazy(Sequence):
    """A read-only sequence whose items are built by ``make(i)`` on first access."""

    def __init__(self, n: int, make):
        self._items: list = [None] * n
        self._make = make

    def __len__(self) -> int:
        return len(self._items)

    def __getitem__(self, i):
        if isinstance(i, slice):
            return [self[j] for j in range(*i.indices(len(self)))]
        item = self._items[i]
        if item is None:
            item = self._items[i] = self._make(i if i >= 0 else i + len(self))
        return item


class PlannedEntry:
    """One reference encode of the batch (the native counterpart of ``EntryRecord``)."""

    __slots__ = ("plan", "index", "row", "uri", "text", "use_memory", "visible", "chunks", "wave", "_metadata")

    def __init__(self, plan: "NativeBatchPlan", i: int):
        out = plan.out
        self.plan, self.index = plan, i
        self.row = int(out["entry_row"][i])
        self.uri = out["entry_uri"][i]
        self.text = out["entry_text"][i]
        self.use_memory = bool(out["entry_use_memory"][i])
        first = plan.rows[self.row][0]
        self.visible = tuple(range(first, i)) if self.use_memory else ()
        self.chunks = list(range(int(out["entry_chunk_begin"][i]), int(out["entry_chunk_end"][i])))
        self.wave = int(out["entry_wave"][i])
        self._metadata = None

    @property
    def metadata(self) -> dict:
        if self._metadata is None:
            local = int(self.plan.out["entry_local"][self.index])
            self._metadata = self.plan.python_row(self.row).entries[local].metadata
        return self._metadata


class PlannedChunk:
    """One routable chunk of the batch (the native counterpart of ``ChunkRecord``)."""

    __slots__ = ("plan", "index", "row", "entry", "uri", "chunk_id", "token_start", "token_end", "seq", "_metadata")

    def __init__(self, plan: "NativeBatchPlan", i: int):
        out = plan.out
        self.plan, self.index = plan, i
        self.entry = int(out["chunk_entry"][i])
        self.row = int(out["entry_row"][self.entry])
        self.uri = out["entry_uri"][self.entry]
        self.chunk_id = chunk_identity(self.uri, int(out["chunk_index"][i]))
        self.token_start = int(out["chunk_start"][i])
        self.token_end = int(out["chunk_end"][i])
        self.seq = int(out["chunk_seq"][i])
        self._metadata = None

    @property
    def token_ids(self) -> tuple:
        off = self.plan.out["chunk_token_off"]
        return tuple(int(t) for t in self.plan.out["tokens"][off[self.index]: off[self.index + 1]])

    @property
    def metadata(self) -> dict:
        if self._metadata is None:
            first_entry = self.plan.rows[self.row][0]
            first_chunk = int(self.plan.out["entry_chunk_begin"][first_entry])
            self._metadata = self.plan.python_row(self.row).chunks[self.index - first_chunk].metadata
        return self._metadata


class PlannedAudit:
    """Resolution events and dependency edges of one row, materialised on first read."""

    def __init__(self, events: list[tuple], dependencies: list[tuple]):
        self._raw = (events, dependencies)
        self._events = self._deps = None

    @property
    def events(self) -> list[ResolutionEvent]:
        if self._events is None:
            self._events = [ResolutionEvent(u, kind, depth, parent, detail) for u, kind, depth, parent, detail in self._raw[0]]
        return self._events

    @property
    def dependencies(self) -> list[dict]:
        if self._deps is None:
            self._deps = [{"parent_uri": p, "child_uri": c, "cyclic": cyc, "action": a} for p, c, cyc, a in self._raw[1]]
        return self._deps


class PlannedCache(PRASimpleMemoryCache):
    """A row's (empty) planning cache whose audit trail is read from a ``PlannedAudit`` on demand."""

    def __init__(self, audit: PlannedAudit):
        super().__init__()
        self._audit = audit

    @property
    def resolution_events(self):
        audit = self.__dict__.get("_audit")
        return audit.events if audit is not None else self.__dict__.get("_events_value", [])

    @resolution_events.setter
    def resolution_events(self, value):
        self.__dict__["_audit"] = None
        self.__dict__["_events_value"] = value

    @property
    def dependencies(self):
        audit = self.__dict__.get("_audit")
        return audit.dependencies if audit is not None else self.__dict__.get("_deps_value", [])

    @dependencies.setter
    def dependencies(self, value):
        self.__dict__["_deps_value"] = value


class NativeBatchPlan:
    """A batch plan made by the native planner, with the attributes of ``BatchPlan``."""

    native = True

    def __init__(self, out: dict, metadata_rows: list, replan):
        self.out = out
        self.metadata_rows = metadata_rows
        self._replan = replan  # row index -> Python RowPlan (metadata on demand)
        self._python_rows: dict = {}
        self.rows = [list(r) for r in out["rows"]]
        self.seq_len = int(out["seq_len"])
        self.waves = [list(w) for w in out["waves"]]
        self.wave_tables = out["wave_tables"]
        self.prompt_table = out["prompt"]
        self.packed = out["packed"]
        self.entries = _Lazy(len(out["entry_row"]), lambda i: PlannedEntry(self, i))
        self.chunks = _Lazy(len(out["chunk_entry"]), lambda i: PlannedChunk(self, i))
        self.builders = [PlannedAudit(ev, dp) for ev, dp in out["audit"]]
        self.caches = [PlannedCache(audit) for audit in self.builders]

    def python_row(self, row: int):
        plan = self._python_rows.get(row)
        if plan is None:
            plan = self._python_rows[row] = self._replan(row)
        return plan

    def fill_kmeans(self, tables) -> None:
        """Write each wave's k-means initialisation offsets (by chunk length) into the packed array."""
        packed = self.packed
        for t in self.wave_tables:
            if "km_first" not in t or not t["n"]:
                continue
            off, n, _ = t["lens"]
            firsts, offs = tables.lookup(packed[off: off + n].tolist())
            f0 = t["km_first"][0]
            o0 = t["km_off"][0]
            packed[f0: f0 + n] = np.asarray(firsts, dtype=np.int32)
            packed[o0: o0 + n] = np.asarray(offs, dtype=np.int32)
