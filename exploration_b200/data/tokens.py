"""Token corpora: a headerless file of native-endian token ids, read in place.

The file is opened as a read-only numpy memory map; a batch is one fancy-index
gather of ``batch x (length + 1)`` ids from the map (only the touched pages
are read) widened to int64, so neither the corpus nor a per-row Python loop
is ever materialised. Nothing is downloaded.

The window starts are drawn with ``torch.randint`` from the caller's
generator in the reference's order (st/data/tokens.py:24-31), so one seed
selects the same windows in both frameworks.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

TOKEN_DTYPES = {"uint8": np.uint8, "uint16": np.uint16, "int32": np.int32, "int64": np.int64}

# The extracted enwik8 file and its standard 90M / 5M / 5M byte split.
ENWIK8_BYTES = 100_000_000
ENWIK8_SPLITS = {"train": (0, 90_000_000), "val": (90_000_000, 95_000_000), "test": (95_000_000, 100_000_000)}


class TokenDataset:
    """Random contiguous windows ``[start, start + length]`` of ids ``[start, stop)`` of a token file."""

    def __init__(self, path, dtype: str = "uint16", start: int = 0, stop: int | None = None):
        if dtype not in TOKEN_DTYPES:
            raise ValueError("token dtype must be uint8/uint16/int32/int64")
        self.path = Path(path)
        item = np.dtype(TOKEN_DTYPES[dtype])
        size = self.path.stat().st_size
        if size % item.itemsize:
            raise ValueError("token file size is not a multiple of the token width")
        count = size // item.itemsize
        stop = count if stop is None else stop
        if not 0 <= start < stop <= count:
            raise ValueError("invalid corpus token interval")
        self._ids = np.memmap(self.path, dtype=item, mode="r", offset=start * item.itemsize, shape=(stop - start,))

    def __len__(self) -> int:
        return self._ids.shape[0]

    def batch(self, batch_size: int, length: int, generator: torch.Generator):
        """``(ids, next ids, all-true mask, None)``, each ``[batch_size, length]``."""
        if len(self) < length + 1:
            raise ValueError(f"corpus has {len(self)} tokens; a window needs {length + 1}")
        starts = torch.randint(len(self) - length, (batch_size,), generator=generator)
        gather = starts.numpy()[:, None] + np.arange(length + 1)
        windows = torch.from_numpy(self._ids[gather].astype(np.int64))
        return windows[:, :-1], windows[:, 1:], torch.ones(batch_size, length, dtype=torch.bool), None


def enwik8_dataset(path="data/enwik8", split: str = "train") -> TokenDataset:
    """One split of the extracted 100,000,000-byte enwik8 file as byte tokens."""
    if split not in ENWIK8_SPLITS:
        raise ValueError("enwik8 split must be train/val/test")
    if Path(path).stat().st_size != ENWIK8_BYTES:
        raise ValueError("enwik8 must be the extracted 100,000,000-byte file")
    return TokenDataset(path, "uint8", *ENWIK8_SPLITS[split])
