"""Tokenisers with atomic ``<REF_n>`` handles (``src/data/tokenizer.py:13-130``).

``PRATokenizer`` is the character tokenizer whose ``stoi``/``itos`` are stored in
checkpoints; ids are assigned to the sorted character set (text plus
``string.printable``) and reference tokens are appended as they appear.
``WordIdTokenizer`` maps whitespace-separated ``t<id>`` words to integer ids; it
is how synthetic uniform-random token streams of a large vocabulary are carried
through the text-based dataset format.
"""

from __future__ import annotations

import re
import string

REF_TOKEN_PATTERN = re.compile(r"<REF_\d+>")


class PRATokenizer:
    """Character tokenizer; unknown characters map to ``?``."""

    def __init__(self, texts: list[str] | None = None, extra_tokens: list[str] | None = None):
        self.stoi: dict[str, int] = {}
        self.itos: dict[int, str] = {}
        joined = "".join(list(texts or []) + list(extra_tokens or ["<REF_0>"]))
        refs = sorted(set(REF_TOKEN_PATTERN.findall(joined)))
        alphabet = sorted(set(REF_TOKEN_PATTERN.sub("", joined)) | set(string.printable))
        self.stoi = {ch: index for index, ch in enumerate(alphabet)}
        for token in refs:
            self.register_reference_token(token)
        self.itos = {index: token for token, index in self.stoi.items()}

    @property
    def vocab_size(self) -> int:
        return len(self.stoi)

    @classmethod
    def from_vocab(cls, stoi: dict[str, int]) -> "PRATokenizer":
        tok = cls([])
        tok.stoi = {str(k): int(v) for k, v in stoi.items()}
        tok.itos = {v: k for k, v in tok.stoi.items()}
        return tok

    def register_reference_token(self, token: str) -> int:
        if not REF_TOKEN_PATTERN.fullmatch(token):
            raise ValueError(f"Invalid reference token: {token}")
        if token not in self.stoi:
            self.stoi[token] = len(self.stoi)
            self.itos[self.stoi[token]] = token
        return self.stoi[token]

    def encode(self, text: str) -> list[int]:
        unknown = self.stoi["?"]
        out: list[int] = []
        cursor = 0
        for match in REF_TOKEN_PATTERN.finditer(text):
            out.extend(self.stoi.get(ch, unknown) for ch in text[cursor:match.start()])
            out.append(self.register_reference_token(match.group(0)))
            cursor = match.end()
        out.extend(self.stoi.get(ch, unknown) for ch in text[cursor:])
        return out

    def decode(self, ids) -> str:
        return "".join(self.itos[int(i)] for i in ids)


class WordIdTokenizer:
    """``"t17 t4 <REF_2>"`` <-> ``[17, 4, ref_id]``: a fixed integer vocabulary.

    Ids ``0..base_vocab-1`` are the words ``t0..t{base_vocab-1}`` (id 0 doubles as
    the pad / ignore id); reference tokens are registered above ``base_vocab``.
    """

    def __init__(self, base_vocab: int, reference_tokens: list[str] | None = None):
        self.base_vocab = int(base_vocab)
        self._refs: dict[str, int] = {}
        self.stoi: dict[str, int] = {f"t{i}": i for i in range(self.base_vocab)}
        self.itos: dict[int, str] = {i: f"t{i}" for i in range(self.base_vocab)}
        for token in reference_tokens or ["<REF_0>"]:
            self.register_reference_token(token)

    def register_reference_token(self, token: str) -> int:
        if not REF_TOKEN_PATTERN.fullmatch(token):
            raise ValueError(f"Invalid reference token: {token}")
        if token not in self._refs:
            index = self.base_vocab + len(self._refs)
            self._refs[token] = index
            self.stoi[token] = index
            self.itos[index] = token
        return self._refs[token]

    @property
    def vocab_size(self) -> int:
        return self.base_vocab + len(self._refs)

    def native_word_ids(self) -> tuple[int, dict[str, int]]:
        """(base vocabulary, registered reference tokens): what a native tokenizer needs to
        encode exactly as ``encode`` does for texts whose reference tokens are registered."""
        return self.base_vocab, dict(self._refs)

    def encode(self, text: str) -> list[int]:
        words = text.split()
        out = list(map(self.stoi.get, words))  # one C-level pass; None marks a word not in stoi
        if None in out:  # unregistered reference handles, non-canonical or unknown words
            for i, value in enumerate(out):
                if value is None:
                    out[i] = self._encode_word(words[i])
        return out

    def _encode_word(self, word: str) -> int:
        if REF_TOKEN_PATTERN.fullmatch(word):
            return self.register_reference_token(word)
        if word.startswith("t") and word[1:].isdigit() and int(word[1:]) < self.base_vocab:
            return int(word[1:])
        return 0

    def decode(self, ids) -> str:
        itos = self.itos
        try:
            return " ".join([itos[i] for i in ids])
        except (KeyError, TypeError):  # tensor elements, or ids above the registered range
            return " ".join(itos.get(i) or f"t{i}" for i in map(int, ids))


class BPETokenizer:
    """Hugging Face ``tokenizers`` BPE behind the PRA tokenizer interface."""

    DEFAULT_SPECIAL_TOKENS = ["[PAD]", "[UNK]", "[BOS]", "[EOS]"]

    def __init__(self, tokenizer):
        self.tokenizer = tokenizer
        self._refresh_vocab()

    @classmethod
    def train(cls, texts, *, vocab_size: int = 2_000, reference_tokens: list[str] | None = None,
              min_frequency: int = 2) -> "BPETokenizer":
        from tokenizers import Tokenizer
        from tokenizers.decoders import BPEDecoder
        from tokenizers.models import BPE
        from tokenizers.pre_tokenizers import Whitespace
        from tokenizers.trainers import BpeTrainer

        tok = Tokenizer(BPE(unk_token="[UNK]"))
        tok.pre_tokenizer = Whitespace()
        tok.decoder = BPEDecoder(suffix="</w>")
        trainer = BpeTrainer(vocab_size=int(vocab_size), min_frequency=int(min_frequency),
                             special_tokens=[*cls.DEFAULT_SPECIAL_TOKENS, *(reference_tokens or [])],
                             end_of_word_suffix="</w>")
        tok.train_from_iterator(texts, trainer=trainer)
        return cls(tok)

    @classmethod
    def from_json(cls, value: str) -> "BPETokenizer":
        from tokenizers import Tokenizer

        return cls(Tokenizer.from_str(value))

    @property
    def vocab_size(self) -> int:
        return self.tokenizer.get_vocab_size()

    @property
    def pad_token_id(self) -> int:
        found = self.tokenizer.token_to_id("[PAD]")
        return 0 if found is None else found

    def _refresh_vocab(self) -> None:
        self.stoi = self.tokenizer.get_vocab()
        self.itos = {v: k for k, v in self.stoi.items()}

    def encode(self, text: str) -> list[int]:
        return self.tokenizer.encode(text).ids

    def decode(self, ids) -> str:
        return self.tokenizer.decode([int(i) for i in ids], skip_special_tokens=False)

    def to_json(self) -> str:
        return self.tokenizer.to_str()
