"""End-to-end parity of the B200 engine against the reference (golden fixtures) and the CPU oracle.

* Teacher-forced logits (all layers over [frames | tokens]) agree with the reference's fp32 logits within
  max-abs 2.5e-2 (bf16 storage between ops, the same rounding points as the reference's Triton path;
  measured 0.013-0.016 for the 7-token vocabulary, 0.023 for the 343-token 4-mer head), and within 1.6x of
  the error the reference's own modules make in bf16 on the same inputs (0.013-0.020,
  tests/golden/make_bf16_logits.py).
* Greedy tokens equal the reference's, per chunk, up to the first step whose fp32 top-2 logit margin is below
  the bf16 noise floor (0.05); from there on a bf16 path may legitimately pick the other token.
* The CUDA-graph decode equals the eager decode token for token.
* At the benchmark size (256 chunks x 2048 frames) the results are batch-invariant (a chunk decodes to the
  same tokens inside the full batch as alone) and agree with the oracle on sampled chunks.
"""

import os

import numpy as np
import pytest
import torch

from golden_io import HERE as GOLDEN, load
from oracle import OracleConfig, OracleModel

pytestmark = pytest.mark.gpu

MARGIN_FLOOR = 0.05
CASES = ["base_theta1e6", "base_theta1e4", "kmer4", "homopolymer", "pos_scale2", "base_b8"]


@pytest.fixture(autouse=True)
def _errors_clear():
    from viktor_b200._lib import check_device_errors
    yield
    torch.cuda.synchronize()
    check_device_errors()


def build(g, B=None, max_new=None, graph=True, max_frames=None):
    from viktor_b200 import Basecaller, DecodeEngine, DecoderConfig
    m = g["meta"]
    model = Basecaller.from_weights(g["weights"], k=m["k"], cfg=DecoderConfig(**m["cfg"]), d_enc=m["d_enc"],
                                    pos_scale=m["pos_scale"])
    eng = DecodeEngine(model, B or len(m["lens"]), max_new or m["max_new"], max_frames or max(m["lens"]),
                       cuda_graph=graph, max_homopolymer=m["max_homopolymer"], device="cuda")
    eng.bias.copy_(torch.from_numpy(g["bias"]))
    return eng


def agree_until_low_margin(got, ref, margin):
    """Per row: True if tokens agree at every step before the first step with margin < floor."""
    ok = []
    for b in range(ref.shape[0]):
        low = np.where(np.nan_to_num(margin[b], nan=np.inf) < MARGIN_FLOOR)[0]
        stop = int(low[0]) if len(low) else ref.shape[1]
        ok.append(np.array_equal(got[b, :stop], ref[b, :stop]))
    return np.array(ok)


def oracle_for(g):
    m = g["meta"]
    return OracleModel(OracleConfig(**m["cfg"]), g["weights"], k=m["k"], pos_scale=m["pos_scale"])


@pytest.mark.parametrize("name", CASES)
def test_teacher_forced_logits_match_reference(name):
    g = load(name)
    m = g["meta"]
    eng = build(g, max_new=g["tf_tokens"].shape[1], graph=False)
    got = eng.teacher_forced_logits(torch.from_numpy(g["frames"]), m["lens"],
                                    torch.from_numpy(g["tf_tokens"])).cpu().numpy()
    err = np.abs(got - g["tf_logits"]).max()
    ref_bf16 = np.abs(np.load(os.path.join(GOLDEN, "ref_bf16_logits.npz"))[name] - g["tf_logits"]).max()
    print(f"{name}: max |logits - reference fp32| = {err:.4f} (the reference's own bf16 path: {ref_bf16:.4f})")
    assert err < 2.5e-2, f"max |logits - reference fp32| = {err}"
    assert err < 1.6 * ref_bf16, f"{err} against the reference's own bf16 error {ref_bf16}"


@pytest.mark.parametrize("name", CASES)
def test_greedy_tokens_match_reference(name):
    g = load(name)
    m = g["meta"]
    eng = build(g)
    got = eng.generate(torch.from_numpy(g["frames"]), m["lens"], m["max_new"]).cpu().numpy()
    _, margin = oracle_for(g).generate(g["frames"], m["lens"], m["max_new"], steps=m["max_new"], bias=g["bias"],
                                       max_homopolymer=m["max_homopolymer"])
    ok = agree_until_low_margin(got, g["tokens"], margin)
    assert ok.all(), f"rows disagreeing before a low-margin step: {np.where(~ok)[0]}\n{got}\n{g['tokens']}"
    exact = (got == g["tokens"]).all(1).mean()
    print(f"{name}: identical rows {exact:.3f}")


def test_graph_equals_eager():
    g = load("base_b8")
    m = g["meta"]
    frames = torch.from_numpy(g["frames"])
    a = build(g, graph=True).generate(frames, m["lens"], m["max_new"]).clone()
    b = build(g, graph=False).generate(frames, m["lens"], m["max_new"]).clone()
    assert torch.equal(a, b)


def test_engine_reuse_and_decode_until_done():
    """A second generate() on the same engine reproduces the first; steps=None stops early once every row
    emitted EOS (default grammar, EOS not masked) and fills the rest with PAD."""
    g = load("base_theta1e4")
    m = g["meta"]
    eng = build(g)
    frames = torch.from_numpy(g["frames"])
    a = eng.generate(frames, m["lens"], m["max_new"]).clone()
    b = eng.generate(frames, m["lens"], m["max_new"]).clone()
    assert torch.equal(a, b)
    c = eng.generate(frames, m["lens"], None).clone()
    assert torch.equal(c, a)


@pytest.fixture(scope="module")
def full_size():
    """The benchmark configuration: 256 chunks of 2048 frames, BASELINE architecture, torch-default init."""
    from viktor_b200 import Basecaller, DecodeEngine, DecoderConfig
    from viktor_b200.synthetic import make_frames, make_weights
    cfg = DecoderConfig(vocab_size=7, rope_theta=1e6)
    weights = make_weights(cfg, seed=21, init="torch")
    lens = [2048] * 256
    frames = make_frames(lens, seed=22)
    model = Basecaller.from_weights(weights, k=1, cfg=cfg)
    steps = 12
    eng = DecodeEngine(model, 256, steps, 2048, max_homopolymer=None, device="cuda")
    eng.bias[2] = float("-inf")
    out = eng.generate(torch.from_numpy(frames), lens, steps).cpu().numpy()
    return dict(weights=weights, frames=frames, lens=lens, out=out, steps=steps, model=model, cfg=cfg, eng=eng)


def test_full_size_batch_invariance(full_size):
    from viktor_b200 import DecodeEngine
    f = full_size
    pick = [0, 77, 200, 255]
    eng = DecodeEngine(f["model"], len(pick), f["steps"], 2048, max_homopolymer=None, device="cuda")
    eng.bias[2] = float("-inf")
    sub = np.concatenate([f["frames"][2048 * b:2048 * (b + 1)] for b in pick])
    got = eng.generate(torch.from_numpy(sub), [2048] * len(pick), f["steps"]).cpu().numpy()
    assert np.array_equal(got, f["out"][pick])


def test_full_size_matches_oracle_on_samples(full_size):
    f = full_size
    pick = [3, 150]
    om = OracleModel(OracleConfig(vocab_size=7, rope_theta=1e6), f["weights"], k=1)
    bias = np.zeros(7, np.float32)
    bias[[0, 1, 2]] = -np.inf
    sub = np.concatenate([f["frames"][2048 * b:2048 * (b + 1)] for b in pick])
    ref, margin = om.generate(sub, [2048] * len(pick), f["steps"], steps=f["steps"], bias=bias, max_homopolymer=None)
    ok = agree_until_low_margin(f["out"][pick], ref, margin)
    assert ok.all(), f"\n{f['out'][pick]}\n{ref}\n{margin}"


def test_greedy_chunks_identical_to_oracle_rate():
    """128 chunks of 64..512 frames, 32 greedy steps against the fp32 oracle, which reproduces the reference's
    fp32 tokens on this case for every chunk (tests/golden/identity_b128.npz).  Every chunk agrees up to its first
    step whose fp32 top-2 margin is below the bf16 noise floor.  Over all 32 steps, with this random (untrained)
    init, a few chunks meet an fp32 near-tie where any bf16 path may pick the other token: the reference's own
    bf16 path (its torch engine with the model in bf16) keeps 121 / 128 chunks = 0.945 identical to its fp32
    tokens, this engine 0.969 (B200).  Held: at least the reference's own bf16 rate, and 0.95."""
    from golden_io import identity_case, load_identity
    from viktor_b200 import Basecaller, DecodeEngine, DecoderConfig
    lens, frames, weights = identity_case()
    fx = load_identity()
    steps = 32
    cfg = DecoderConfig(vocab_size=7, rope_theta=1e6)
    model = Basecaller.from_weights(weights, k=1, cfg=cfg)
    eng = DecodeEngine(model, len(lens), steps, max(lens), max_homopolymer=None, device="cuda")
    eng.bias[2] = float("-inf")
    got = eng.generate(torch.from_numpy(frames), lens, steps).cpu().numpy()
    bias = np.zeros(7, np.float32)
    bias[[0, 1, 2]] = -np.inf
    om = OracleModel(OracleConfig(vocab_size=7, rope_theta=1e6), weights, k=1)
    ref, margin = om.generate(frames, lens, steps, steps=steps, bias=bias, max_homopolymer=None)
    assert np.array_equal(ref, fx["tokens_fp32"]), "oracle == reference fp32 tokens on this case"
    ok = agree_until_low_margin(got, ref, margin)
    exact = (got == ref).all(1).mean()
    ref_bf16 = (fx["tokens_bf16"] == fx["tokens_fp32"]).all(1).mean()
    print(f"identical chunks {exact:.4f} ({(got == ref).all(1).sum()} / {len(lens)}); the reference's own bf16 "
          f"path: {ref_bf16:.4f}")
    assert ok.all(), np.where(~ok)[0]
    assert exact >= ref_bf16 and exact >= 0.95


def test_sub_batches_groups_and_empty_prefix():
    """Prefill in sub-batches of 2 (last one partial), a chunk with no frames, 1 / 2 / 3 decode groups (uneven
    row ranges): the same tokens everywhere, and the oracle's up to each chunk's first low-margin step."""
    from viktor_b200 import Basecaller, DecodeEngine, DecoderConfig
    g = load("base_b8")
    m = g["meta"]
    lens = [5, 0, 64, 31, 200]
    from viktor_b200.synthetic import make_frames
    frames = make_frames(lens, seed=44)
    model = Basecaller.from_weights(g["weights"], k=m["k"], cfg=DecoderConfig(**m["cfg"]), d_enc=m["d_enc"])
    outs = []
    for groups, pb in ((1, 128), (2, 2), (3, 2)):
        eng = DecodeEngine(model, len(lens), 20, max(lens), prefill_batch=pb, max_homopolymer=None, device="cuda",
                           decode_groups=groups)
        eng.bias[2] = float("-inf")
        outs.append(eng.generate(torch.from_numpy(frames), lens, 20).cpu().numpy())
    assert all(np.array_equal(o, outs[0]) for o in outs[1:])
    bias = np.zeros(7, np.float32)
    bias[[0, 1, 2]] = -np.inf
    ref, margin = oracle_for(g).generate(frames, lens, 20, steps=20, bias=bias, max_homopolymer=None)
    ok = agree_until_low_margin(outs[0], ref, margin)
    assert ok.all(), f"\n{outs[0]}\n{ref}"


def test_generate_again_with_other_lengths():
    """A second generate() with different prefix lengths (new prefill plan, longer and shorter rows) gives the
    tokens a fresh engine gives."""
    from viktor_b200 import Basecaller, DecodeEngine, DecoderConfig
    from viktor_b200.synthetic import make_frames
    g = load("base_b8")
    m = g["meta"]
    model = Basecaller.from_weights(g["weights"], k=m["k"], cfg=DecoderConfig(**m["cfg"]), d_enc=m["d_enc"])
    a_lens, b_lens = [40, 7, 300], [300, 1, 120]
    fa, fb = make_frames(a_lens, seed=45), make_frames(b_lens, seed=46)
    eng = DecodeEngine(model, 3, 16, 300, max_homopolymer=None, device="cuda")
    eng.bias[2] = float("-inf")
    eng.generate(torch.from_numpy(fa), a_lens, 16)
    got = eng.generate(torch.from_numpy(fb), b_lens, 16).cpu().numpy()
    fresh = DecodeEngine(model, 3, 16, 300, max_homopolymer=None, device="cuda")
    fresh.bias[2] = float("-inf")
    ref = fresh.generate(torch.from_numpy(fb), b_lens, 16).cpu().numpy()
    assert np.array_equal(got, ref)


def test_pinned_host_frames_equal_device_frames():
    """Frames in pinned host memory (copied per prefill sub-batch on a copy stream, overlapping the previous
    sub-batch's prefill) and pageable host frames give the tokens of device-resident frames."""
    from viktor_b200 import Basecaller, DecodeEngine, DecoderConfig
    from viktor_b200.synthetic import make_frames
    g = load("base_b8")
    m = g["meta"]
    model = Basecaller.from_weights(g["weights"], k=m["k"], cfg=DecoderConfig(**m["cfg"]), d_enc=m["d_enc"])
    lens = [100, 37, 256, 3, 180]
    frames = torch.from_numpy(make_frames(lens, seed=47))
    eng = DecodeEngine(model, len(lens), 12, 256, prefill_batch=2, max_homopolymer=None, device="cuda")
    eng.bias[2] = float("-inf")
    ref = eng.generate(frames.cuda(), lens, 12).clone()
    pinned = eng.generate(frames.pin_memory(), lens, 12).clone()
    pageable = eng.generate(frames, lens, 12).clone()
    assert torch.equal(pinned, ref) and torch.equal(pageable, ref)


def test_engine_from_a_model_built_from_the_reference_checkpoint_map():
    """DecodeEngine built from a model assembled only from the reference's state-dict names and shapes
    (tests/golden/reference_state_dict.json, recorded from the stock viktor.Basecaller) decodes exactly as one
    built from this package's Basecaller with the same weights."""
    from test_checkpoint import MAP, reference_like_model
    from viktor_b200 import Basecaller, DecodeEngine, DecoderConfig
    from viktor_b200.synthetic import make_frames, make_weights
    for key, k in (("k1", 1), ("k4", 4)):
        cfg = DecoderConfig(vocab_size=MAP[key]["vocab_size"], rope_theta=1e6)
        weights = make_weights(cfg, seed=31 + k, init="torch")
        lens = [64, 200, 1, 130]
        frames = torch.from_numpy(make_frames(lens, seed=33))
        outs = []
        for model in (reference_like_model(MAP[key]["params"], k, weights).cuda(),
                      Basecaller.from_weights(weights, k=k, cfg=cfg)):
            model.decoder.cfg = cfg
            eng = DecodeEngine(model, len(lens), 16, max(lens), max_homopolymer=None, device="cuda")
            eng.bias[2] = float("-inf")
            outs.append(eng.generate(frames, lens, 16).clone())
        assert torch.equal(outs[0], outs[1])
