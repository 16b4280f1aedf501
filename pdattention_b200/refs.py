"""Reference-token parsing helpers (``src/pra_torch/refs.py:1-93``)."""

import re
import warnings
from dataclasses import dataclass

from .core.references import ReferenceHandle, ReferenceTable

LEGACY_REF_PATTERN = re.compile(r"!!ref:(?P<uri>[^!]+)!!")
REF_TOKEN_PATTERN = re.compile(r"<REF_(?P<id>\d+)>")


@dataclass(frozen=True)
class RefHandle:
    """A located legacy ``!!ref:uri!!`` marker."""

    raw: str
    uri: str
    start: int
    end: int


@dataclass(frozen=True)
class ReferenceTokenOccurrence:
    """A located ``<REF_n>`` token and its optional table binding."""

    token: str
    id: int
    start: int
    end: int
    handle: ReferenceHandle | None = None


def parse_refs(text: str) -> list[RefHandle]:
    warnings.warn("parse_refs() supports deprecated !!ref:uri!! syntax; use parse_ref_tokens() with a "
                  "ReferenceTable.", DeprecationWarning, stacklevel=2)
    return [RefHandle(m.group(0), m.group("uri"), m.start(), m.end()) for m in LEGACY_REF_PATTERN.finditer(text)]


def parse_ref_tokens(text: str, reference_table: ReferenceTable | None = None) -> list[ReferenceTokenOccurrence]:
    out = []
    for m in REF_TOKEN_PATTERN.finditer(text):
        token = m.group(0)
        bound = reference_table.find_by_token(token) if reference_table else None
        out.append(ReferenceTokenOccurrence(token, int(m.group("id")), m.start(), m.end(), bound))
    return out


def normalize_ref_tokens(text: str, ref_token: str | None = None) -> str:
    return LEGACY_REF_PATTERN.sub("<REF>" if ref_token is None else ref_token, text)


def split_uri_anchor(uri: str) -> tuple[str, str | None]:
    base, sep, anchor = uri.partition("#")
    return (base, anchor or None) if sep else (uri, None)


def parent_anchor(anchor: str | None) -> str | None:
    if not anchor or "." not in anchor:
        return None
    return anchor.rsplit(".", 1)[0]


def child_anchor(anchor: str | None, child: str) -> str:
    return f"{anchor}.{child}" if anchor else child
