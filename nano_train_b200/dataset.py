"""Datasets and loaders (reference: src/dataset.py:24-133).

``TextDataset(text_path, max_seq_length)``: character-level vocabulary with
id 0 reserved for ``<pad>``, overlapping windows of ``max_seq_length``
characters at stride ``max_seq_length // 2``, items
``{"input_ids": seq[:-1], "labels": seq[1:]}`` with padding labels set to
-100. ``create_dataloader(dataset, batch_size, shuffle, sampler)``.
``SyntheticTokenDataset`` gives seeded uniform token ids for benchmarks.
"""
from __future__ import annotations

from pathlib import Path
from typing import Optional, TypedDict

import torch
from torch.utils.data import DataLoader, Dataset, RandomSampler, Sampler

from .logging import get_logger

logger = get_logger(__name__)


class Batch(TypedDict):
    input_ids: torch.Tensor
    labels: torch.Tensor


class TextDataset(Dataset):
    def __init__(self, text_path: str, max_seq_length: int = 256) -> None:
        if max_seq_length < 2:
            raise ValueError("max_seq_length must be at least 2")
        path = Path(text_path)
        if not path.exists():
            raise FileNotFoundError(f"Dataset file not found: {text_path}")
        text = path.read_text(encoding="utf-8")
        self.max_seq_length = max_seq_length
        self.pad_token, self.pad_id = "<pad>", 0
        self.chars = [self.pad_token] + sorted(set(text))
        self.vocab_size = len(self.chars)
        self.char_to_idx = {c: i for i, c in enumerate(self.chars)}
        self.idx_to_char = dict(enumerate(self.chars))
        ids = torch.tensor([self.char_to_idx[c] for c in text], dtype=torch.long)
        stride = max(1, max_seq_length // 2)
        starts = range(0, max(0, ids.numel() - max_seq_length + 1), stride)
        self.sequences = [ids[s:s + max_seq_length] for s in starts]
        if not self.sequences and ids.numel() > 0:
            pad = torch.full((max_seq_length - ids.numel(),), self.pad_id, dtype=torch.long)
            self.sequences = [torch.cat([ids[:max_seq_length], pad])]
        logger.info("TextDataset: %d chars, vocab %d, %d sequences", ids.numel(), self.vocab_size,
                    len(self.sequences))

    def __len__(self) -> int:
        return len(self.sequences)

    def __getitem__(self, idx: int) -> Batch:
        seq = self.sequences[idx]
        if seq.numel() < self.max_seq_length:
            seq = torch.cat([seq, torch.full((self.max_seq_length - seq.numel(),), self.pad_id, dtype=torch.long)])
        labels = seq[1:].clone()
        labels[labels == self.pad_id] = -100
        return {"input_ids": seq[:-1].clone(), "labels": labels}

    def decode(self, ids) -> str:
        return "".join(self.idx_to_char.get(int(i), "") for i in ids)


class SyntheticTokenDataset(Dataset):
    """``num_samples`` sequences of seeded uniform token ids (labels = next token)."""

    def __init__(self, num_samples: int, seq_len: int, vocab_size: int, seed: int = 0) -> None:
        g = torch.Generator().manual_seed(seed)
        self.data = torch.randint(0, vocab_size, (num_samples, seq_len + 1), generator=g)

    def __len__(self) -> int:
        return self.data.shape[0]

    def __getitem__(self, i: int) -> Batch:
        row = self.data[i]
        return {"input_ids": row[:-1].clone(), "labels": row[1:].clone()}


def create_dataloader(dataset: Dataset, batch_size: int, shuffle: bool = True,
                      sampler: Optional[Sampler] = None, pin_memory: bool = False) -> DataLoader:
    if batch_size <= 0:
        raise ValueError("batch_size must be positive")
    return DataLoader(dataset, batch_size=batch_size, shuffle=bool(shuffle) and sampler is None, sampler=sampler,
                      num_workers=0, drop_last=False, pin_memory=pin_memory)


class EpochSeedRandomSampler(RandomSampler):
    """A shuffling sampler whose order is exactly that of ``RandomSampler`` without a generator:
    each epoch's seed is drawn from the global torch RNG when iteration starts (so a run follows
    the same batch order as the reference's ``DataLoader(shuffle=True)``). The drawn seed is kept
    in ``epoch_seed``; ``force_next_seed`` makes the next epoch reuse a recorded seed without
    drawing, which is how a resumed run continues the interrupted epoch in the same order."""

    def __init__(self, data_source) -> None:
        super().__init__(data_source)
        self.epoch_seed: Optional[int] = None
        self._forced: Optional[int] = None

    def force_next_seed(self, seed: Optional[int]) -> None:
        self._forced = None if seed is None else int(seed)

    def __iter__(self):
        if self._forced is not None:
            seed, self._forced = self._forced, None
        else:
            seed = int(torch.empty((), dtype=torch.int64).random_().item())
        self.epoch_seed = seed
        self.generator = torch.Generator().manual_seed(seed)
        try:
            yield from super().__iter__()
        finally:
            self.generator = None

