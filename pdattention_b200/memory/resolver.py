"""URI resolution: the boundary between PRA routing and wherever content lives.

``InMemoryResolver`` serves documents from dictionaries (the contract of
``src/pra_torch/resolver.py:11-95``): a URI, or failing that its anchor-free
base (``doc#section`` -> ``doc``), maps to its text, a local ``<REF_n>`` -> child
URI table, anchors, metadata, version and summary; an unknown URI raises
``KeyError``.  A document value is either plain text or a structured dict whose
fields override the resolver-wide side tables (``summaries``,
``reference_tables``, ``metadata``, ``versions``).
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


def _optional_str(value) -> str | None:
    return None if value is None else str(value)


class InMemoryResolver:
    def __init__(self, documents: dict, summaries: dict[str, str] | None = None,
                 reference_tables: dict[str, dict[str, str]] | None = None, metadata: dict[str, dict] | None = None,
                 versions: dict[str, str] | None = None):
        self.documents = dict(documents)
        self.summaries = summaries or {}
        self.reference_tables = reference_tables or {}
        self.metadata = metadata or {}
        self.versions = versions or {}

    def _document(self, uri: str):
        for key in dict.fromkeys((uri, split_uri_anchor(uri)[0])):
            value = self.documents.get(key)
            if value is not None:
                return value
        raise KeyError(f"Reference URI is not available: {uri}")

    def _fields(self, uri: str, value) -> tuple:
        """(text, table, anchors, metadata, version, summary) of a stored value; side tables are
        keyed by the requested URI and fill whatever a structured value leaves out."""
        side_table = self.reference_tables.get(uri) or {}
        side_meta = self.metadata.get(uri, {})
        if not isinstance(value, dict):
            return (str(value), dict(side_table), {}, dict(side_meta), self.versions.get(uri),
                    self.summaries.get(uri))
        return (str(value.get("text", "")), dict(value.get("reference_table") or side_table),
                dict(value.get("anchors") or {}), {**side_meta, **dict(value.get("metadata") or {})},
                value.get("version", self.versions.get(uri)), value.get("summary", self.summaries.get(uri)))

    def resolve(self, uri: str, summary_only: bool = False) -> ResolvedReference:
        """The document behind ``uri``; ``summary_only`` returns the summary as the text."""
        text, table, anchors, metadata, version, summary = self._fields(uri, self._document(uri))
        return ResolvedReference(uri=uri, text=str(summary or "") if summary_only else text,
                                 reference_table={str(token): str(child) for token, child in table.items()},
                                 anchors=anchors, metadata=metadata, version=_optional_str(version),
                                 summary=_optional_str(summary))

    def resolve_handle(self, handle: ReferenceHandle, summary_only: bool = False) -> HandleResolvedReference:
        """The handle-oriented view: children as unnumbered handles (id -1) in table order."""
        resolved = self.resolve(handle.uri, summary_only=summary_only)
        return HandleResolvedReference(
            handle=handle, text=resolved.text,
            children=[ReferenceHandle(id=-1, token=token, uri=child) for token, child in resolved.reference_table.items()],
            metadata={**resolved.metadata, "version": resolved.version})
