"""The raw logits file of zeninfer's `logits --out F.bin` (src/main.cpp:505-511):
the float32 logits [S][V] of S positions, little-endian, back to back, no header
(the format tools/check_logits.py reads).  Lets logits from the real model feed the
sampler's tests and benchmark instead of the synthetic workloads."""

from __future__ import annotations

import os

import numpy as np

QWEN25_VOCAB = 151936


def read_logits(path: str, n_vocab: int = QWEN25_VOCAB, mmap: bool = True) -> np.ndarray:
    """float32 [S, n_vocab] view of a logits file (memory-mapped by default)."""
    size = os.path.getsize(path)
    if n_vocab <= 0 or size % (4 * n_vocab) != 0:
        raise ValueError(f"{path}: {size} bytes is not a whole number of {n_vocab}-float rows")
    rows = size // (4 * n_vocab)
    if mmap:
        return np.memmap(path, dtype="<f4", mode="r", shape=(rows, n_vocab))
    return np.fromfile(path, dtype="<f4").reshape(rows, n_vocab)


def write_logits(path: str, logits: np.ndarray) -> None:
    """Writes [S, V] (or [V]) logits in the same format."""
    np.ascontiguousarray(logits, dtype="<f4").tofile(path)
