"""Loader wrapper with the reference's 80/10/10 seeded split (``src/data/datamodules.py``).

Adds rank-aware sharding for data-parallel training: with ``world_size > 1``
each rank iterates a disjoint ``DistributedSampler`` shard of the train split.
"""

import torch
from torch.utils.data import DataLoader, DistributedSampler, random_split

from .collators import PRACollator
from .datasets import PRADataset, dataset_class_for_stage
from .tokenizer import PRATokenizer


class PRADataModule:
    def __init__(self, dataset_stage: str, data_dir: str = "data", max_examples: int | None = None,
                 batch_size: int = 8, max_seq_len: int = 96, shuffle: bool = True, num_workers: int = 0,
                 pin_memory: bool = False, persistent_workers: bool = False, tokenizer=None, split_seed: int = 0,
                 rank: int = 0, world_size: int = 1):
        self.dataset_stage = dataset_stage
        self.data_dir = data_dir
        self.max_examples = max_examples
        self.batch_size = batch_size
        self.max_seq_len = max_seq_len
        self.shuffle = shuffle
        self.num_workers = num_workers
        self.pin_memory = pin_memory
        self.persistent_workers = persistent_workers and num_workers > 0
        self.tokenizer = tokenizer
        self.split_seed = int(split_seed)
        self.rank, self.world_size = int(rank), int(world_size)
        self.dataset: PRADataset | None = None
        self.train_dataset = self.val_dataset = self.test_dataset = None
        self.collator: PRACollator | None = None

    def load(self):
        self.dataset = dataset_class_for_stage(self.dataset_stage)(self.data_dir, max_examples=self.max_examples)
        if self.tokenizer is None:
            self.tokenizer = PRATokenizer(self._corpus(self.dataset))
        self.collator = PRACollator(self.tokenizer, max_seq_len=self.max_seq_len)
        self.train_dataset, self.val_dataset, self.test_dataset = self._split(self.dataset, seed=self.split_seed)
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
        sampler = None
        if shard and self.world_size > 1:
            sampler = DistributedSampler(dataset, num_replicas=self.world_size, rank=self.rank, shuffle=shuffle,
                                         seed=self.split_seed)
            shuffle = False
        return DataLoader(dataset, batch_size=self.batch_size, shuffle=shuffle, sampler=sampler,
                          num_workers=self.num_workers, pin_memory=self.pin_memory,
                          persistent_workers=self.persistent_workers, collate_fn=self.collator)

    @staticmethod
    def _corpus(dataset) -> list[str]:
        texts = []
        for sample in dataset:
            texts.append(sample.question + " " + sample.answer)
            for ref in sample.references:
                texts.append(ref.summary or "")
                texts.append(str(ref.metadata.get("text", "")))
        return texts

    @staticmethod
    def _split(dataset, *, seed: int = 0):
        n = len(dataset)
        if n < 3:
            return dataset, dataset, dataset
        n_train, n_val = max(1, int(n * 0.8)), max(1, int(n * 0.1))
        n_test = n - n_train - n_val
        if n_test <= 0:
            n_test = 1
            n_train = n - n_val - n_test
        return random_split(dataset, [n_train, n_val, n_test], generator=torch.Generator().manual_seed(seed))
