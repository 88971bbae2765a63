"""Generate ``ref_bf16_logits.npz``: the REFERENCE's teacher-forced logits computed in bf16.

For every golden case with the product's shapes (tests/golden_io.CASES minus the sampled ones, which share
their logits path), the reference's ``Basecaller.logits`` (viktor/model.py:55-60) runs on CPU with its modules
in bf16 — bf16 storage between ops, as in the reference's bf16 inference path — on the same inputs as the
case's fp32 ``tf_logits``.  Only ``lm_head`` stays fp32: ``logits`` hands the head an fp32 hidden state
(viktor/model.py:60).  The stored arrays (one per case, ``<name>``, fp32) give the error the reference's own
bf16 path makes against its fp32 logits; the GPU test of the engine's teacher-forced logits holds the engine's
error to the same scale.

Usage:  python tests/golden/make_bf16_logits.py --reference PATH_TO_VIKTOR_CHECKOUT
"""

from __future__ import annotations

import argparse
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))  # the repository (viktor_b200)
sys.path.insert(0, os.path.dirname(HERE))  # tests/ (golden_io)
from golden_io import load  # noqa: E402

CASES = ["base_theta1e6", "base_theta1e4", "kmer4", "homopolymer", "pos_scale2", "base_b8"]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("VIKTOR_REFERENCE"))
    args = ap.parse_args()
    if not args.reference:
        ap.error("pass --reference or set VIKTOR_REFERENCE")
    sys.dont_write_bytecode = True
    sys.path.insert(0, args.reference)
    import torch
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    from viktor import Basecaller, DecoderConfig, KmerTokenizer

    out = {}
    for name in CASES:
        g = load(name)
        m = g["meta"]
        tok = KmerTokenizer(m["k"])
        model = Basecaller(types.SimpleNamespace(d_model=m["d_enc"]), tok, DecoderConfig(**m["cfg"])).eval()
        model.load_state_dict({n: torch.from_numpy(a) for n, a in g["weights"].items()}, strict=True)
        model.pos_scale = m["pos_scale"]
        model = model.to(torch.bfloat16)
        model.decoder.lm_head.float()
        lens = m["lens"]
        offs = np.concatenate([[0], np.cumsum(lens)])
        with torch.no_grad():
            logits = np.stack([
                model.logits(torch.from_numpy(g["frames"][offs[b]:offs[b + 1]]).to(torch.bfloat16)[None],
                             torch.from_numpy(g["tf_tokens"][b])[None])[0].float().numpy()
                for b in range(len(lens))])
        out[name] = logits.astype(np.float32)
        print(f"{name}: reference bf16 vs fp32 max |logits| error {np.abs(logits - g['tf_logits']).max():.4f}")
    np.savez_compressed(os.path.join(HERE, "ref_bf16_logits.npz"), **out)


if __name__ == "__main__":
    main()
