"""The data-parallel runner with real engines (the reference's scripts/evaluate.py:127-138 pattern): spawned
worker processes each build a DecodeEngine on their strided shard of the chunks and decode it; the parent merges
the token arrays.  With one GPU both workers share it (independent processes, no kernel waits on another), so the
test runs on the driver's single-GPU box; the merged tokens must equal one engine decoding every chunk."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LENS = [300, 17, 256, 1, 128, 64, 200, 90, 33]
STEPS = 20


def _model():
    from golden_io import load
    from viktor_b200 import Basecaller, DecoderConfig
    g = load("base_b8")
    m = g["meta"]
    return Basecaller.from_weights(g["weights"], k=m["k"], cfg=DecoderConfig(**m["cfg"]), d_enc=m["d_enc"])


def decode_shard(rank, world, indices, device_index):
    """Worker: decode the chunks `indices` on cuda:device_index (EOS masked, fixed steps); returns host tokens."""
    import os
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    sys.path.insert(0, os.path.dirname(here))
    from viktor_b200 import DecodeEngine
    from viktor_b200.synthetic import make_frames
    torch.cuda.set_device(device_index)
    lens = [LENS[i] for i in indices]
    frames = make_frames(LENS, seed=49)
    offs = np.concatenate([[0], np.cumsum(LENS)])
    mine = np.concatenate([frames[offs[i]:offs[i + 1]] for i in indices])
    eng = DecodeEngine(_model(), len(lens), STEPS, max(LENS), max_homopolymer=None, device=f"cuda:{device_index}")
    eng.bias[2] = float("-inf")
    out = eng.generate(torch.from_numpy(mine), lens, STEPS).cpu().numpy()
    eng.check_errors()
    return out


def test_run_sharded_with_engines_equals_one_engine():
    from viktor_b200 import DecodeEngine
    from viktor_b200.parallel import merge_shards, run_sharded
    from viktor_b200.synthetic import make_frames
    parts = run_sharded(decode_shard, len(LENS), 2, args=(0,), timeout=600)
    merged = merge_shards(parts, len(LENS))
    eng = DecodeEngine(_model(), len(LENS), STEPS, max(LENS), max_homopolymer=None, device="cuda")
    eng.bias[2] = float("-inf")
    whole = eng.generate(torch.from_numpy(make_frames(LENS, seed=49)), LENS, STEPS).cpu().numpy()
    assert np.array_equal(merged, whole)
