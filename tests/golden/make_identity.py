"""Generate ``identity_b128.npz``: the REFERENCE's own greedy tokens in fp32 and in bf16 on one case.

The case is ``golden_io.identity_case()``, the one of the engine's identity-rate test (tests/test_gpu_engine.py):
128 chunks of 64..512 frames, untrained ``init="torch"`` weights, vocabulary 7, rope theta 1e6, EOS masked, no
homopolymer stop, 32 greedy steps.  The reference package ``viktor`` (GHSSHG/Viktor) runs it on CPU through its
stock ``DecodeEngine(backend="torch")`` twice: with the model in fp32 and with the model in bf16 (the reference's
engine computes in its weights' dtype, viktor/engine.py:38).  Stored: both token arrays and the lengths.  The fraction of chunks whose bf16 tokens equal
the fp32 tokens over all 32 steps is the identity rate the reference itself reaches in bf16 with this
(untrained) init; the GPU test holds this package's bf16 engine to the same measure.

Usage:  python tests/golden/make_identity.py --reference PATH_TO_VIKTOR_CHECKOUT
"""

from __future__ import annotations

import argparse
import os
import sys
import time
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))  # the repository (viktor_b200)
sys.path.insert(0, os.path.dirname(HERE))  # tests/ (golden_io)
from golden_io import identity_case  # noqa: E402

STEPS = 32


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
    from viktor import Basecaller, DecodeEngine, DecoderConfig, KmerTokenizer
    from viktor.tokenizer import EOS

    lens, frames, weights = identity_case()
    tok = KmerTokenizer(1)
    out = {}
    for name, dtype in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
        model = Basecaller(types.SimpleNamespace(d_model=512), tok,
                           DecoderConfig(vocab_size=tok.vocab_size, rope_theta=1e6)).eval()
        model.load_state_dict({n: torch.from_numpy(a) for n, a in weights.items()}, strict=True)
        model = model.to(dtype)
        t0 = time.time()
        with torch.no_grad():
            eng = DecodeEngine(model, len(lens), STEPS, max(lens), backend="torch", cuda_graph=False,
                               max_homopolymer=None)
            eng.bias[EOS] = float("-inf")
            out[name] = eng.generate(torch.from_numpy(frames).to(dtype), lens, STEPS).clone().numpy()
        print(f"{name}: {time.time() - t0:.1f} s", flush=True)
    same = (out["fp32"] == out["bf16"]).all(1)
    print(f"reference bf16 vs fp32: identical chunks {same.mean():.4f} ({same.sum()} / {len(lens)})")
    np.savez_compressed(os.path.join(HERE, "identity_b128.npz"), tokens_fp32=out["fp32"].astype(np.int8),
                        tokens_bf16=out["bf16"].astype(np.int8), lens=np.array(lens, np.int32))


if __name__ == "__main__":
    main()
