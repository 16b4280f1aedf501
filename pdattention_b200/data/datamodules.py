"""Stage data module: dataset, tokenizer, collator and train/val/test loaders.

Public surface of ``src/data/datamodules.py:9-108`` (constructor arguments,
``load`` / ``train_loader`` / ``val_loader`` / ``test_loader`` /
``build_reference_tables``).  The split is the reference's seeded 80/10/10
``random_split`` (so a seed selects the same examples in both frameworks); a
character tokenizer, when none is given, is fitted to every question, answer,
reference summary and reference text.  For data-parallel training
(``world_size > 1``) the train loader iterates this rank's disjoint
``DistributedSampler`` shard, reshuffled per epoch with ``sampler.set_epoch``.
"""

from __future__ import annotations

import torch
from torch.utils.data import DataLoader, DistributedSampler, random_split

from .collators import PRACollator
from .datasets import PRADataset, dataset_class_for_stage
from .tokenizer import PRATokenizer


def split_sizes(n: int) -> tuple[int, int, int] | None:
    """(train, val, test) sizes of ``n`` examples, or ``None`` when every split is the whole set."""
    if n < 3:
        return None
    val = max(1, int(n * 0.1))
    train = max(1, int(n * 0.8))
    test = n - train - val
    return (train, val, test) if test > 0 else (n - val - 1, val, 1)


def tokenizer_corpus(dataset) -> list[str]:
    """Texts a fitted character vocabulary must cover."""
    texts = []
    for sample in dataset:
        texts.append(f"{sample.question} {sample.answer}")
        texts.extend(piece for ref in sample.references
                     for piece in (ref.summary or "", str(ref.metadata.get("text", ""))))
    return texts


class PRADataModule:
    def __init__(self, dataset_stage: str, data_dir: str = "data", max_examples: int | None = None,
                 batch_size: int = 8, max_seq_len: int = 96, shuffle: bool = True, num_workers: int = 0,
                 pin_memory: bool = False, persistent_workers: bool = False, tokenizer=None, split_seed: int = 0,
                 rank: int = 0, world_size: int = 1):
        self.dataset_stage, self.data_dir, self.max_examples = dataset_stage, data_dir, max_examples
        self.batch_size, self.max_seq_len, self.shuffle = batch_size, max_seq_len, shuffle
        self.num_workers, self.pin_memory = num_workers, pin_memory
        self.persistent_workers = bool(persistent_workers and num_workers > 0)
        self.tokenizer = tokenizer
        self.split_seed = int(split_seed)
        self.rank, self.world_size = int(rank), int(world_size)
        self.dataset: PRADataset | None = None
        self.collator: PRACollator | None = None
        self._splits: dict[str, object] = {}

    # split datasets (None before load())
    train_dataset = property(lambda self: self._splits.get("train"))
    val_dataset = property(lambda self: self._splits.get("val"))
    test_dataset = property(lambda self: self._splits.get("test"))

    def load(self):
        self.dataset = dataset_class_for_stage(self.dataset_stage)(self.data_dir, max_examples=self.max_examples)
        self.tokenizer = self.tokenizer or PRATokenizer(tokenizer_corpus(self.dataset))
        self.collator = PRACollator(self.tokenizer, max_seq_len=self.max_seq_len)
        sizes = split_sizes(len(self.dataset))
        parts = ([self.dataset] * 3 if sizes is None else
                 random_split(self.dataset, list(sizes), generator=torch.Generator().manual_seed(self.split_seed)))
        self._splits = dict(zip(("train", "val", "test"), parts))
        return self

    def train_loader(self) -> DataLoader:
        return self._loader(self.train_dataset, shuffle=self.shuffle, shard=True)

    def val_loader(self) -> DataLoader:
        return self._loader(self.val_dataset, shuffle=False)

    def test_loader(self) -> DataLoader:
        return self._loader(self.test_dataset, shuffle=False)

    def build_reference_tables(self):
        if self.dataset is None:
            self.load()
        return [self.dataset.build_reference_table(sample) for sample in self.dataset]

    def _loader(self, dataset, shuffle: bool, shard: bool = False) -> DataLoader:
        if dataset is None:
            raise RuntimeError("PRADataModule.load() must be called before requesting loaders.")
        sampler = (DistributedSampler(dataset, num_replicas=self.world_size, rank=self.rank, shuffle=shuffle,
                                      seed=self.split_seed) if shard and self.world_size > 1 else None)
        return DataLoader(dataset, batch_size=self.batch_size, shuffle=shuffle and sampler is None, sampler=sampler,
                          num_workers=self.num_workers, pin_memory=self.pin_memory,
                          persistent_workers=self.persistent_workers, collate_fn=self.collator)

    # kept for callers of the reference's private helpers
    _corpus = staticmethod(tokenizer_corpus)

    @staticmethod
    def _split(dataset, *, seed: int = 0):
        sizes = split_sizes(len(dataset))
        if sizes is None:
            return dataset, dataset, dataset
        return random_split(dataset, list(sizes), generator=torch.Generator().manual_seed(seed))
