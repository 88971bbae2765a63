"""Loads the golden fixtures and rebuilds their seeded inputs (shared by CPU and GPU tests)."""

import json
import os

import numpy as np

from viktor_b200.config import DecoderConfig
from viktor_b200.synthetic import make_frames, make_weights

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = ["base_theta1e6", "base_theta1e4", "kmer4", "homopolymer", "pos_scale2", "base_b8", "tiny", "sampled_t07",
         "sampled_kmer4"]
SAMPLED = ["sampled_t07", "sampled_kmer4"]


def load(name):
    z = np.load(os.path.join(HERE, f"{name}.npz"))
    meta = json.loads(str(z["meta"]))
    cfg = DecoderConfig(**meta["cfg"])
    if any(k.startswith("w:") for k in z.files):
        weights = {k[2:]: z[k] for k in z.files if k.startswith("w:")}
    else:
        weights = make_weights(cfg, seed=meta["weight_seed"], init=meta["init"], d_enc=meta["d_enc"])
    frames = make_frames(meta["lens"], d_enc=meta["d_enc"], seed=meta["frame_seed"])
    meta.setdefault("temperature", 0.0)
    return dict(meta=meta, cfg=cfg, weights=weights, frames=frames, tokens=z["tokens"],
                tf_logits=z["tf_logits"], tf_tokens=z["tf_tokens"], bias=z["bias"],
                noise=z["noise"] if "noise" in z.files else None)


def identity_case():
    """The 128-chunk case of the identity-rate tests: lengths, frames, weights (vocabulary 7, theta 1e6)."""
    rng = np.random.default_rng(32)
    lens = [int(v) for v in rng.integers(64, 513, 128)]
    weights = make_weights(DecoderConfig(vocab_size=7, rope_theta=1e6), seed=31, init="torch")
    return lens, make_frames(lens, seed=33), weights


def load_identity():
    """identity_b128.npz (tests/golden/make_identity.py): the reference's greedy tokens on identity_case(), with
    the model in fp32 and in bf16, 32 steps, EOS masked."""
    z = np.load(os.path.join(HERE, "identity_b128.npz"))
    return dict(tokens_fp32=z["tokens_fp32"].astype(np.int64), tokens_bf16=z["tokens_bf16"].astype(np.int64),
                lens=[int(v) for v in z["lens"]])
