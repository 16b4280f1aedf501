"""QuestionSample batches -> padded tensors plus reference metadata (``src/data/collators.py``).

Layout contract kept from the reference: the sequence is ``prompt + " answer\\n"``,
labels are next-token ids masked with the pad id (0) before the answer, and the
pad id doubles as the loss ``ignore_index``.  The untruncated ids/labels are kept
in metadata for implicit ``#__head`` prompts.
"""

from dataclasses import asdict

import torch

from ..core.references import ReferenceTable
from .schemas import QuestionSample


class PRACollator:
    def __init__(self, tokenizer, max_seq_len: int, pad_token_id: int = 0):
        self.tokenizer = tokenizer
        self.max_seq_len = max_seq_len
        self.pad_token_id = pad_token_id

    def _row(self, sample: QuestionSample):
        pad = self.pad_token_id
        prompt = self.tokenizer.encode(sample.question)
        answer = self.tokenizer.encode(" " + sample.answer.strip() + "\n")
        full = prompt + answer
        full_labels = full[1:] + [pad]
        head = max(len(prompt) - 1, 0)
        full_labels[:head] = [pad] * head
        ids = full[: self.max_seq_len]
        labels = (ids[1:] + [pad])[: len(ids)]
        masked = max(min(len(prompt), len(ids)) - 1, 0)
        labels[:masked] = [pad] * masked
        return prompt, full, full_labels, ids, labels

    def __call__(self, samples: list[QuestionSample]) -> dict:
        inputs, labels, masks, tables, metadata = [], [], [], [], []
        for sample in samples:
            prompt, full, full_labels, ids, row_labels = self._row(sample)
            inputs.append(torch.tensor(ids, dtype=torch.long))
            labels.append(torch.tensor(row_labels, dtype=torch.long))
            masks.append(torch.ones(len(ids), dtype=torch.long))
            tables.append(self._build_reference_table(sample))
            metadata.append({
                "id": sample.id,
                "question": sample.question,
                "answer": sample.answer,
                "references": sample.references,
                "target_reference_ids": sample.target_reference_ids,
                "target_reference_uris": sample.target_reference_uris
                or sample.metadata.get("target_reference_uris", []),
                "target_chunk_ids": sample.target_chunk_ids or sample.metadata.get("target_chunk_ids", []),
                "target_chunk_spans": sample.target_chunk_spans or sample.metadata.get("target_chunk_spans", []),
                "expected_anchors": sample.metadata.get("expected_anchors", []),
                "full_input_ids": tuple(full),
                "full_labels": tuple(full_labels),
                "prompt_token_count": len(prompt),
                "sample": sample,
                "asdict": asdict(sample),
            })
        return {
            "input_ids": self._pad(inputs, self.pad_token_id),
            "labels": self._pad(labels, self.pad_token_id),
            "attention_mask": self._pad(masks, 0),
            "reference_tables": tables,
            "metadata": metadata,
        }

    @staticmethod
    def _build_reference_table(sample: QuestionSample) -> ReferenceTable:
        table = ReferenceTable()
        for ref in sample.references:
            table.register(uri=ref.uri, summary=ref.summary, metadata=ref.metadata, id=ref.id,
                           token=f"<REF_{ref.id}>")
        return table

    @staticmethod
    def _pad(rows: list[torch.Tensor], value: int) -> torch.Tensor:
        width = max(int(r.numel()) for r in rows)
        out = torch.full((len(rows), width), value, dtype=rows[0].dtype)
        for i, r in enumerate(rows):
            out[i, : r.numel()] = r
        return out
