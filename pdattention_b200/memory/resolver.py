"""URI resolution boundary (``src/pra_torch/resolver.py:11-95``).

A resolver maps a URI (or its anchor-free base) to content, a local
``<REF_n>`` -> child URI table, anchors, metadata, version and summary, and
raises ``KeyError`` for unknown URIs.
"""

from __future__ import annotations

from dataclasses import dataclass, field

from ..core.references import ReferenceHandle, ResolvedReference as HandleResolvedReference
from ..refs import split_uri_anchor


@dataclass
class ResolvedReference:
    uri: str
    text: str
    reference_table: dict[str, str] = field(default_factory=dict)
    anchors: dict[str, str] = field(default_factory=dict)
    metadata: dict = field(default_factory=dict)
    version: str | None = None
    summary: str | None = None


class InMemoryResolver:
    """Dictionary-backed resolver; values are strings or structured dicts."""

    def __init__(self, documents: dict, summaries: dict[str, str] | None = None,
                 reference_tables: dict[str, dict[str, str]] | None = None, metadata: dict[str, dict] | None = None,
                 versions: dict[str, str] | None = None):
        self.documents = dict(documents)
        self.summaries = summaries or {}
        self.reference_tables = reference_tables or {}
        self.metadata = metadata or {}
        self.versions = versions or {}

    def _lookup(self, uri: str):
        value = self.documents.get(uri)
        if value is None:
            value = self.documents.get(split_uri_anchor(uri)[0])
        if value is None:
            raise KeyError(f"Reference URI is not available: {uri}")
        return value

    def resolve(self, uri: str, summary_only: bool = False) -> ResolvedReference:
        value = self._lookup(uri)
        if isinstance(value, dict):
            text = str(value.get("text", ""))
            table = dict(value.get("reference_table") or self.reference_tables.get(uri) or {})
            anchors = dict(value.get("anchors") or {})
            meta = {**self.metadata.get(uri, {}), **dict(value.get("metadata") or {})}
            version = value.get("version", self.versions.get(uri))
            summary = value.get("summary", self.summaries.get(uri))
        else:
            text, table, anchors = str(value), dict(self.reference_tables.get(uri) or {}), {}
            meta, version, summary = dict(self.metadata.get(uri, {})), self.versions.get(uri), self.summaries.get(uri)
        return ResolvedReference(
            uri=uri, text=str(summary or "") if summary_only else text,
            reference_table={str(k): str(v) for k, v in table.items()}, anchors=anchors, metadata=meta,
            version=str(version) if version is not None else None,
            summary=str(summary) if summary is not None else None)

    def resolve_handle(self, handle: ReferenceHandle, summary_only: bool = False) -> HandleResolvedReference:
        resolved = self.resolve(handle.uri, summary_only=summary_only)
        children = [ReferenceHandle(id=-1, token=t, uri=u) for t, u in resolved.reference_table.items()]
        return HandleResolvedReference(handle=handle, text=resolved.text, children=children,
                                       metadata={**resolved.metadata, "version": resolved.version})
