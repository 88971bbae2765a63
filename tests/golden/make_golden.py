"""Generate the golden fixtures of this directory by running the REFERENCE implementation.

Imports the reference package ``viktor`` (GHSSHG/Viktor) from a checkout named by ``--reference`` or the
``VIKTOR_REFERENCE`` environment variable, runs it on CPU in fp32 and stores its outputs as small ``.npz``
files.  Inputs are not stored: weights and frames are regenerated from seeds by
``viktor_b200.synthetic`` (numpy only), so the tests rebuild identical inputs anywhere.

Each fixture holds, for one model configuration:
  * ``tokens``      reference greedy tokens, ``DecodeEngine(backend="torch").generate``
                    (viktor/engine.py:168-220); sampled tokens for the cases with a temperature
  * ``noise``       (sampled cases) the uniform draws [max_new, B, V] that stood in for ``torch.rand_like`` in
                    the reference's selection (viktor/engine.py:82), one per selected token, seeded
  * ``tf_logits``   teacher-forced logits per chunk, ``Basecaller.logits`` (viktor/model.py:55-60)
  * ``tf_tokens``   the teacher-forcing inputs used for them ([BOS] + seeded tokens)
  * ``meta``        JSON: config, seeds, lengths, engine settings
The ``tiny`` fixture also stores its weights (a few KB), since its shapes are not the product's.

Usage:  python tests/golden/make_golden.py --reference PATH_TO_VIKTOR_CHECKOUT
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from viktor_b200.config import DecoderConfig as OurConfig  # noqa: E402
from viktor_b200.synthetic import make_frames, make_weights  # noqa: E402

# name -> settings.  "cfg" overrides DecoderConfig defaults; vocab follows k.
CASES = {
    # BASELINE architecture, rope theta 1e6; EOS masked so sequences keep running
    "base_theta1e6": dict(k=1, cfg=dict(rope_theta=1e6), lens=[5, 33, 64], max_new=24, mask_eos=True,
                          max_homopolymer=None, weight_seed=0, frame_seed=1, tf_len=12),
    # the reference decoder's default theta (viktor/decoder.py:34) and the default grammar
    "base_theta1e4": dict(k=1, cfg=dict(rope_theta=1e4), lens=[17, 48], max_new=16, mask_eos=False,
                          max_homopolymer=64, weight_seed=3, frame_seed=4, tf_len=10),
    # 4-mer vocabulary (343): tail tokens force EOS, then PAD
    "kmer4": dict(k=4, cfg=dict(rope_theta=1e6), lens=[7, 40, 21], max_new=20, mask_eos=True,
                  max_homopolymer=None, weight_seed=5, frame_seed=6, tf_len=8),
    # homopolymer stop: a bias on 'A' makes the run reach max_homopolymer
    "homopolymer": dict(k=1, cfg=dict(rope_theta=1e6), lens=[9, 30], max_new=12, mask_eos=True,
                        max_homopolymer=5, bias_add={3: 30.0}, weight_seed=7, frame_seed=8, tf_len=6),
    # RoPE positions rescaled for the prefix (viktor/model.py:37-40, viktor/engine.py:55,159,197)
    "pos_scale2": dict(k=1, cfg=dict(rope_theta=1e6), lens=[12, 50], max_new=12, mask_eos=True,
                       max_homopolymer=None, pos_scale=2, weight_seed=9, frame_seed=10, tf_len=8),
    # larger batch for token agreement on the GPU
    "base_b8": dict(k=1, cfg=dict(rope_theta=1e6), lens=[1, 64, 127, 128, 129, 200, 255, 300], max_new=40,
                    mask_eos=True, max_homopolymer=None, weight_seed=11, frame_seed=12, tf_len=16),
    # sampled decoding (viktor/engine.py:81-82): Gumbel-perturbed argmax at temperature 0.7 / 1.0
    "sampled_t07": dict(k=1, cfg=dict(rope_theta=1e6), lens=[9, 40, 23], max_new=16, mask_eos=False,
                        max_homopolymer=64, weight_seed=15, frame_seed=16, tf_len=6, temperature=0.7, noise_seed=17),
    "sampled_kmer4": dict(k=4, cfg=dict(rope_theta=1e6), lens=[14, 31], max_new=14, mask_eos=False,
                          max_homopolymer=64, weight_seed=18, frame_seed=19, tf_len=6, temperature=1.0,
                          noise_seed=20),
    # the reference's own unit-test model shape (tests/test_viktor.py:25-30): oracle generality only
    "tiny": dict(k=4, cfg=dict(d_model=32, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=8, ffn_dim=64,
                              max_seq_len=512), d_enc=32, lens=[64, 128, 64], max_new=20, mask_eos=False,
                 max_homopolymer=64, weight_seed=13, frame_seed=14, tf_len=10, store_weights=True),
}


def run_case(name, c, viktor):
    import torch
    from viktor import Basecaller, DecodeEngine, DecoderConfig, KmerTokenizer
    from viktor.tokenizer import EOS

    tok = KmerTokenizer(c["k"])
    cfg_kw = dict(vocab_size=tok.vocab_size, **c["cfg"])
    d_enc = c.get("d_enc", 512)
    weights = make_weights(OurConfig(**cfg_kw), seed=c["weight_seed"], init="torch", d_enc=d_enc)
    model = Basecaller(types.SimpleNamespace(d_model=d_enc), tok, DecoderConfig(**cfg_kw)).eval()
    model.load_state_dict({n: torch.from_numpy(a) for n, a in weights.items()}, strict=True)
    model.pos_scale = c.get("pos_scale", 1)
    lens = c["lens"]
    frames = make_frames(lens, d_enc=d_enc, seed=c["frame_seed"])
    B = len(lens)
    T = c.get("temperature", 0.0)
    noise = None
    rand_like = torch.rand_like
    if T > 0:
        noise = np.random.default_rng(c["noise_seed"]).random((c["max_new"], B, tok.vocab_size), dtype=np.float32)
        drawn = [0]

        def seeded_rand_like(t, **kw):  # the reference's only random draw: one [B, V] per selection
            assert tuple(t.shape) == (B, tok.vocab_size)
            u = torch.from_numpy(noise[drawn[0]].copy())
            drawn[0] += 1
            return u

        torch.rand_like = seeded_rand_like
    with torch.no_grad():
        eng = DecodeEngine(model, B, c["max_new"], max(lens), backend="torch", cuda_graph=False,
                           max_homopolymer=c["max_homopolymer"], temperature=T)
        if c["mask_eos"]:
            eng.bias[EOS] = float("-inf")
        for t, v in c.get("bias_add", {}).items():
            eng.bias[int(t)] += v
        tokens = eng.generate(torch.from_numpy(frames), lens, c["max_new"]).clone().numpy()
        torch.rand_like = rand_like
        if T > 0:
            assert drawn[0] == c["max_new"]
        bias = eng.bias.numpy().copy()
        rng = np.random.default_rng(c["frame_seed"] + 1000)
        tf_tokens = np.concatenate([np.ones((B, 1), np.int64),
                                    rng.integers(3, tok.vocab_size, (B, c["tf_len"] - 1))], 1)
        offs = np.concatenate([[0], np.cumsum(lens)])
        tf_logits = np.stack([
            model.logits(torch.from_numpy(frames[offs[b]:offs[b + 1]])[None],
                         torch.from_numpy(tf_tokens[b])[None])[0].numpy() for b in range(B)])
    meta = dict(name=name, k=c["k"], cfg=cfg_kw, d_enc=d_enc, lens=lens, max_new=c["max_new"],
                mask_eos=c["mask_eos"], max_homopolymer=c["max_homopolymer"], pos_scale=c.get("pos_scale", 1),
                bias_add=c.get("bias_add", {}), weight_seed=c["weight_seed"], frame_seed=c["frame_seed"],
                init="torch", temperature=T)
    arrays = dict(tokens=tokens, tf_logits=tf_logits.astype(np.float32), tf_tokens=tf_tokens,
                  bias=bias.astype(np.float32), meta=np.array(json.dumps(meta)))
    if noise is not None:
        arrays["noise"] = noise
    if c.get("store_weights"):
        arrays.update({"w:" + n: a for n, a in weights.items()})
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)
    print(f"{name}: tokens {tokens.shape} tf_logits {tf_logits.shape}  first row {tokens[0][:12].tolist()}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("VIKTOR_REFERENCE"),
                    help="path of a GHSSHG/Viktor checkout (the directory holding the viktor/ package)")
    ap.add_argument("--only", nargs="*")
    args = ap.parse_args()
    if not args.reference:
        ap.error("pass --reference or set VIKTOR_REFERENCE")
    sys.dont_write_bytecode = True
    sys.path.insert(0, args.reference)
    import torch
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    import viktor
    for name, c in CASES.items():
        if args.only and name not in args.only:
            continue
        run_case(name, c, viktor)


if __name__ == "__main__":
    main()
