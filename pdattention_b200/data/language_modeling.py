"""Plain causal-LM data (``src/data/language_modeling.py``): fixed token blocks."""

from __future__ import annotations

import torch
from torch.utils.data import DataLoader, Dataset


class TokenBlockDataset(Dataset):
    """Concatenate token ids and cut them into ``block_size + 1`` windows."""

    def __init__(self, token_ids: list[int], block_size: int, max_blocks: int | None = None):
        self.block_size = int(block_size)
        span = self.block_size + 1
        count = max(len(token_ids) - 1, 0) // self.block_size
        if max_blocks is not None:
            count = min(count, int(max_blocks))
        self.blocks = [token_ids[i * self.block_size: i * self.block_size + span] for i in range(count)]
        self.blocks = [b for b in self.blocks if len(b) == span]

    def __len__(self) -> int:
        return len(self.blocks)

    def __getitem__(self, index: int) -> dict:
        block = torch.tensor(self.blocks[index], dtype=torch.long)
        return {"input_ids": block[:-1], "labels": block[1:]}


def collate_blocks(rows: list[dict]) -> dict:
    ids = torch.stack([r["input_ids"] for r in rows])
    return {"input_ids": ids, "labels": torch.stack([r["labels"] for r in rows]),
            "attention_mask": torch.ones_like(ids)}


class WikiTextDataModule:
    """Token blocks over WikiText (needs the ``datasets`` package and a local cache)."""

    def __init__(self, tokenizer, block_size: int = 128, batch_size: int = 8, dataset_name: str = "wikitext-2-raw-v1",
                 max_train_documents: int | None = None, max_eval_documents: int | None = None,
                 max_train_blocks: int | None = None, cache_dir=None):
        self.tokenizer = tokenizer
        self.block_size = block_size
        self.batch_size = batch_size
        self.dataset_name = dataset_name
        self.max_train_documents = max_train_documents
        self.max_eval_documents = max_eval_documents
        self.max_train_blocks = max_train_blocks
        self.cache_dir = cache_dir
        self.splits: dict[str, TokenBlockDataset] = {}

    @classmethod
    def from_texts(cls, tokenizer, splits: dict[str, list[str]], **kwargs) -> "WikiTextDataModule":
        module = cls(tokenizer, **kwargs)
        module._build(splits)
        return module

    def _build(self, texts: dict[str, list[str]]) -> None:
        for name, docs in texts.items():
            ids = [t for doc in docs for t in self.tokenizer.encode(doc)]
            limit = self.max_train_blocks if name == "train" else None
            self.splits[name] = TokenBlockDataset(ids, self.block_size, limit)

    def load(self):
        from .datasets import load_wikitext_splits, wikitext_documents

        raw = load_wikitext_splits(self.dataset_name, cache_dir=self.cache_dir)
        self._build({
            "train": wikitext_documents(raw["train"], max_documents=self.max_train_documents),
            "validation": wikitext_documents(raw["validation"], max_documents=self.max_eval_documents),
            "test": wikitext_documents(raw["test"], max_documents=self.max_eval_documents),
        })
        return self

    def _loader(self, name: str, shuffle: bool) -> DataLoader:
        return DataLoader(self.splits[name], batch_size=self.batch_size, shuffle=shuffle, collate_fn=collate_blocks)

    def train_loader(self) -> DataLoader:
        return self._loader("train", True)

    def val_loader(self) -> DataLoader:
        return self._loader("validation", False)

    def test_loader(self) -> DataLoader:
        return self._loader("test", False)
