"""Decoder hyperparameters and the token vocabulary.

``DecoderConfig`` keeps the field names and defaults of viktor/decoder.py:25-36 so that a
reference config (or a training snapshot's args) maps onto it one to one.  The vocabulary
layout follows viktor/tokenizer.py:10-54: PAD, BOS, EOS, then every full k-mer in
lexicographic ACGT order, then the tails of length 1..k-1; a tail may only be the last token
before EOS.
"""

from __future__ import annotations

from dataclasses import dataclass
from itertools import product

import numpy as np

PAD, BOS, EOS = 0, 1, 2
N_SPECIAL = 3
BASES = "ACGT"


@dataclass
class DecoderConfig:
    vocab_size: int
    d_model: int = 512
    n_layers: int = 8
    n_heads: int = 8
    n_kv_heads: int = 2
    head_dim: int = 64
    ffn_dim: int = 1536
    rope_theta: float = 10000.0
    norm_eps: float = 1e-6
    max_seq_len: int = 4096


class KmerTokenizer:
    """Output vocabulary of k-mer tokens (viktor/tokenizer.py:16-54)."""

    def __init__(self, k: int):
        self.k = k
        full = ["".join(p) for p in product(BASES, repeat=k)]
        tails = ["".join(p) for n in range(1, k) for p in product(BASES, repeat=n)]
        self.strings = ["<pad>", "<bos>", "<eos>"] + full + tails
        self.ids = {s: i for i, s in enumerate(self.strings) if i >= N_SPECIAL}
        self.vocab_size = len(self.strings)
        self.n_full = len(full)
        tail = np.zeros(self.vocab_size, dtype=bool)
        tail[N_SPECIAL + self.n_full:] = True
        self.tail_mask = tail
        self.n_bases = np.array([0] * N_SPECIAL + [len(s) for s in full + tails], dtype=np.int64)
        # homopolymer full k-mers (AAAA, CCCC, ...): a run of them ends in a forced EOS
        self.homo_mask = np.array([i >= N_SPECIAL and len(s) == k and len(set(s)) == 1
                                   for i, s in enumerate(self.strings)], dtype=bool)

    def encode(self, seq: str) -> list[int]:
        k = self.k
        return [self.ids[seq[i:i + k]] for i in range(0, len(seq), k)]

    def decode(self, ids) -> str:
        out = []
        for i in ids:
            i = int(i)
            if i == EOS:
                break
            if i >= N_SPECIAL:
                out.append(self.strings[i])
        return "".join(out)


def get_tokenizer(name: str) -> KmerTokenizer:
    return {"base": KmerTokenizer(1), "4mer": KmerTokenizer(4)}[name]
