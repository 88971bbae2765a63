"""Records the parameter names and shapes of the REFERENCE model (GHSSHG/Viktor ``viktor.Basecaller``) into
``reference_state_dict.json``, so that the tests can check, without the reference present, that this package
reads exactly the checkpoint keys a reference model carries (viktor/model.py:27-48, viktor/decoder.py:54-134).

The reference ``Basecaller`` holds its encoder as a submodule; the hot path starts after the encoder, so the
map is taken with a stand-in encoder object that only provides ``d_model`` (it registers no parameters), and it
lists the ``projector.*`` and ``decoder.*`` entries of ``state_dict()`` — the keys a snapshot stores under
"projector" and "decoder" (scripts/evaluate.py:107-108).  Buffers that are not persistent (RoPE tables) are
not in a state dict and are not listed.

Usage:  python tests/golden/make_state_dict_map.py --reference PATH_TO_VIKTOR_CHECKOUT
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import types

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("VIKTOR_REFERENCE"))
    args = ap.parse_args()
    if not args.reference:
        sys.exit("give --reference PATH (a GHSSHG/Viktor checkout) or set VIKTOR_REFERENCE")
    sys.path.insert(0, args.reference)
    from viktor import Basecaller, DecoderConfig, KmerTokenizer

    out = {}
    for k in (1, 4):
        tok = KmerTokenizer(k)
        model = Basecaller(types.SimpleNamespace(d_model=512), tok, DecoderConfig(vocab_size=tok.vocab_size))
        sd = model.state_dict()
        out[f"k{k}"] = {"vocab_size": tok.vocab_size,
                        "params": {n: list(t.shape) for n, t in sd.items()},
                        "dtypes": sorted({str(t.dtype) for t in sd.values()})}
    path = os.path.join(HERE, "reference_state_dict.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
    print(path, {k: len(v["params"]) for k, v in out.items()})


if __name__ == "__main__":
    main()
