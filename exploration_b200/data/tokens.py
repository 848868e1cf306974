"""Flat token corpora read through a memory map.

A corpus is a headerless file of native-endian token ids. Nothing is
downloaded and the corpus is never copied whole into int64: a batch slices
the mapped file and widens only the slices it uses
(reference: st/data/tokens.py:6-41).
"""
from __future__ import annotations

from pathlib import Path

import torch

TOKEN_DTYPES = {"uint8": torch.uint8, "uint16": torch.uint16,
                "int32": torch.int32, "int64": torch.int64}

ENWIK8_BYTES = 100_000_000
ENWIK8_SPLITS = {"train": (0, 90_000_000), "val": (90_000_000, 95_000_000),
                 "test": (95_000_000, 100_000_000)}


class TokenDataset:
    """Random contiguous windows from a mapped token file."""

    def __init__(self, path, dtype: str = "uint16", start: int = 0, stop: int | None = None):
        if dtype not in TOKEN_DTYPES:
            raise ValueError("token dtype must be uint8/uint16/int32/int64")
        self.path = Path(path)
        torch_dtype = TOKEN_DTYPES[dtype]
        width = torch.empty((), dtype=torch_dtype).element_size()
        size = self.path.stat().st_size
        if size % width:
            raise ValueError("token file size is not a multiple of the token width")
        total = size // width
        stop = total if stop is None else stop
        if not 0 <= start < stop <= total:
            raise ValueError("invalid corpus token interval")
        mapped = torch.from_file(str(self.path), shared=False, size=total, dtype=torch_dtype)
        self.tokens = mapped[start:stop]

    def __len__(self) -> int:
        return len(self.tokens)

    def batch(self, batch_size: int, length: int, generator: torch.Generator):
        if len(self.tokens) < length + 1:
            raise ValueError(f"corpus has {len(self.tokens)} tokens; a window needs {length + 1}")
        starts = torch.randint(len(self.tokens) - length, (batch_size,), generator=generator)
        windows = torch.stack([self.tokens[int(s):int(s) + length + 1].to(torch.int64)
                               for s in starts])
        return windows[:, :-1], windows[:, 1:], torch.ones(batch_size, length, dtype=torch.bool), None


def enwik8_dataset(path="data/enwik8", split: str = "train") -> TokenDataset:
    """The standard 90M/5M/5M byte split of the extracted enwik8 file."""
    if split not in ENWIK8_SPLITS:
        raise ValueError("enwik8 split must be train/val/test")
    if Path(path).stat().st_size != ENWIK8_BYTES:
        raise ValueError("enwik8 must be the extracted 100,000,000-byte file")
    lo, hi = ENWIK8_SPLITS[split]
    return TokenDataset(path, "uint8", lo, hi)
