"""Synthetic tasks and memory-mapped token corpora."""
from .synthetic import (FILL0, FILL1, KEY, MQAR_FILL0, MQAR_FILL1, MQAR_KEYS, P, Q, SEP, VOCAB,
                        copying_batch, mqar_batch, passkey_batch, random_batch, resolve_npairs)
from .tokens import TokenDataset, enwik8_dataset

__all__ = ["FILL0", "FILL1", "KEY", "MQAR_FILL0", "MQAR_FILL1", "MQAR_KEYS", "P", "Q", "SEP",
           "VOCAB", "copying_batch", "mqar_batch", "passkey_batch", "random_batch",
           "resolve_npairs", "TokenDataset", "enwik8_dataset"]
