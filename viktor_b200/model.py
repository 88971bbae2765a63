"""Basecaller container: per-frame projector + decoder + tokenizer (viktor/model.py:27-48).

Only the parts the inference hot path reads are kept: ``projector`` (Linear(d_enc, d) - GELU - Linear(d, d),
viktor/model.py:35), ``decoder``, ``tokenizer``, ``pos_scale`` and ``cfg``.  The encoder is out of scope; the
engine is fed encoder frames.  ``DecodeEngine`` equally accepts the reference's own ``Basecaller``.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn as nn

from .config import DecoderConfig, KmerTokenizer, get_tokenizer
from .decoder import Decoder


class Basecaller(nn.Module):
    def __init__(self, tokenizer: KmerTokenizer, cfg: DecoderConfig | None = None, d_enc: int = 512):
        super().__init__()
        self.tokenizer = tokenizer
        self.cfg = cfg or DecoderConfig(vocab_size=tokenizer.vocab_size)
        d = self.cfg.d_model
        self.d_enc = d_enc
        self.projector = nn.Sequential(nn.Linear(d_enc, d), nn.GELU(), nn.Linear(d, d))
        self.decoder = Decoder(self.cfg)
        self.pos_scale = 1

    @classmethod
    def from_args(cls, args: dict, d_enc: int = 512):
        """The model of a training run's args (viktor/model.py:42-48): tokenizer, depth, prefix_pos_scale."""
        tok = get_tokenizer(args.get("tokenizer", "base"))
        m = cls(tok, DecoderConfig(vocab_size=tok.vocab_size, n_layers=args.get("layers", 8)), d_enc)
        m.pos_scale = args.get("prefix_pos_scale", 1)
        return m

    @classmethod
    def from_weights(cls, weights: dict, k: int = 1, cfg: DecoderConfig | None = None, d_enc: int = 512,
                     pos_scale: int = 1):
        """Builds the container from a flat state dict (numpy or torch), keyed like the reference model."""
        tok = KmerTokenizer(k)
        m = cls(tok, cfg or DecoderConfig(vocab_size=tok.vocab_size), d_enc)
        sd = {n: torch.from_numpy(np.ascontiguousarray(a)) if isinstance(a, np.ndarray) else a
              for n, a in weights.items()}
        m.load_state_dict(sd, strict=True)
        m.pos_scale = pos_scale
        return m.eval()
