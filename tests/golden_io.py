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
