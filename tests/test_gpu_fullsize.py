"""Parity at the benchmark sizes (configs 2, 3 and 4 of the benchmark), on sampled rows.

The engine decodes the whole batch at the benchmark shape on the GPU; a sample of its rows is decoded again by
the pinned PyTorch CPU port of the reference (oracle/decoder_torch.py, fp32, tokens equal to the reference's on
every golden case).  Weights use the PyTorch-default init (the benchmark's N(0, 0.02) init is degenerate
for token parity).  Rule, as in the golden-case tests: every sampled row agrees with the fp32 tokens
up to its first step whose fp32 top-2 margin is below the bf16 noise floor (0.05); the share of rows identical
over all steps is printed (with this untrained init some rows meet an fp32 near-tie, where any bf16 path may
take the other token).

* config 2: 256 chunks x 2048 frames, 256 greedy steps (EOS masked), 16 rows spread over the batch and both
  decode groups.
* config 3: 512 chunks of U{128..2048 step 128} frames through prefill sub-batches of 128, each chunk decoding
  round(256 x frames / 2048) tokens and then EOS (engine.max_tokens; finished rows take the one-position
  attention shortcut); sampled: the shortest and longest chunks and the rows on either side of every sub-batch
  boundary.  The port has no per-row cap: its tokens past a row's cap are replaced by EOS then PAD.
* config 4: 1024 chunks x 2048 frames, 4-mer vocabulary (343) with the default grammar (tail -> EOS, homopolymer
  stop, PAD after EOS), 280 steps; sampled: rows whose output ends with a tail followed by EOS, and fixed rows.
"""

import numpy as np
import pytest
import torch

from oracle import OracleConfig
from oracle.decoder_torch import TorchCPUModel

pytestmark = pytest.mark.gpu

MARGIN_FLOOR = 0.05
PAD, EOS = 0, 2


@pytest.fixture(autouse=True)
def _errors_clear():
    from viktor_b200._lib import check_device_errors
    yield
    torch.cuda.synchronize()
    check_device_errors()


def _frames(lens, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn(sum(lens), 512, generator=g, device="cuda")


def _rows(frames, lens, rows):
    offs = np.concatenate([[0], np.cumsum(lens)])
    return torch.cat([frames[int(offs[r]):int(offs[r + 1])] for r in rows]).cpu().numpy()


def _compare(got, ref, margin, caps=None):
    """Per row: the first step at which the comparison stops (a low fp32 margin before the row's cap) and
    whether the tokens agree before it.  Steps at or past a row's cap are deterministic (EOS, then PAD) and are
    compared in full."""
    ok, identical, stops = [], [], []
    for i in range(ref.shape[0]):
        m = np.nan_to_num(margin[i], nan=np.inf).copy()
        if caps is not None:
            m[caps[i]:] = np.inf
        low = np.where(m < MARGIN_FLOOR)[0]
        stop = int(low[0]) if len(low) else ref.shape[1]
        stops.append(stop)
        ok.append(np.array_equal(got[i, :stop], ref[i, :stop]))
        identical.append(np.array_equal(got[i], ref[i]))
    return np.array(ok), np.array(identical), np.array(stops)


def _report(name, ok, identical, stops, steps):
    print(f"{name}: {ok.sum()} / {len(ok)} sampled rows agree up to their first low-margin step "
          f"(median stop {int(np.median(stops))} of {steps}); identical over all steps: {identical.mean():.3f}")


def _model(V, k, seed):
    from viktor_b200 import Basecaller, DecoderConfig
    from viktor_b200.synthetic import make_weights
    cfg = DecoderConfig(vocab_size=V, rope_theta=1e6)
    weights = make_weights(cfg, seed=seed, init="torch")
    port = TorchCPUModel(OracleConfig(vocab_size=V, rope_theta=1e6), weights, k=k)
    return Basecaller.from_weights(weights, k=k, cfg=cfg), port


def test_config2_full_size_sampled_rows():
    from viktor_b200 import DecodeEngine
    B, steps = 256, 256
    model, port = _model(7, 1, seed=21)
    lens = [2048] * B
    frames = _frames(lens, seed=22)
    eng = DecodeEngine(model, B, steps, 2048, max_homopolymer=None, device="cuda")
    eng.bias[EOS] = float("-inf")
    got = eng.generate(frames, lens, steps).cpu().numpy()
    pick = list(range(0, B, 17))[:16]
    bias = np.zeros(7, np.float32)
    bias[[0, 1, 2]] = -np.inf
    ref, margin = port.generate(_rows(frames, lens, pick), [2048] * len(pick), steps, bias, None, return_margin=True)
    ok, identical, stops = _compare(got[pick], ref, margin)
    _report("config 2", ok, identical, stops, steps)
    assert ok.all(), f"rows {np.array(pick)[~ok]} disagree before a low-margin step"


def test_config3_varlen_sub_batches_and_decode_lengths():
    from viktor_b200 import DecodeEngine
    from viktor_b200.synthetic import varlen_prefix_lengths
    B, steps = 512, 256
    model, port = _model(7, 1, seed=23)
    lens = varlen_prefix_lengths(B, seed=24)
    caps = [int(round(steps * n / 2048)) for n in lens]
    frames = _frames(lens, seed=25)
    eng = DecodeEngine(model, B, steps, 2048, prefill_batch=128, max_homopolymer=None, device="cuda")
    eng.bias[EOS] = float("-inf")
    eng.max_tokens.copy_(torch.tensor(caps))
    got = eng.generate(frames, lens, None).cpu().numpy()  # stops once every chunk has ended
    pick = sorted({int(np.argmin(lens)), int(np.argmax(lens)), 0, 127, 128, 255, 256, 383, 384, B - 1})
    bias = np.zeros(7, np.float32)
    bias[[0, 1, 2]] = -np.inf
    ref, margin = port.generate(_rows(frames, lens, pick), [lens[r] for r in pick], steps, bias, None,
                                return_margin=True)
    pc = [caps[r] for r in pick]
    for i, c in enumerate(pc):  # the cap: EOS in column c, PAD after
        if c < steps:
            ref[i, c] = EOS
            ref[i, c + 1:] = PAD
    ok, identical, stops = _compare(got[pick], ref, margin, caps=pc)
    _report("config 3", ok, identical, stops, steps)
    assert ok.all(), f"rows {np.array(pick)[~ok]} disagree before a low-margin step"
    # every row of the batch: bases up to its cap, then EOS and PAD
    for b in range(B):
        c = caps[b]
        assert (got[b, :min(c, steps)] >= 3).all()
        if c < steps:
            assert got[b, c] == EOS and (got[b, c + 1:] == PAD).all()


def test_config4_kmer_head_grammar_sampled_rows():
    from viktor_b200 import DecodeEngine
    from viktor_b200.config import KmerTokenizer
    B, steps = 1024, 280
    model, port = _model(343, 4, seed=26)
    lens = [2048] * B
    frames = _frames(lens, seed=27)
    eng = DecodeEngine(model, B, steps, 2048, device="cuda")  # default grammar: EOS allowed, homopolymer stop 64
    got = eng.generate(frames, lens, steps).cpu().numpy()
    tail = np.asarray(KmerTokenizer(4).tail_mask, dtype=bool)
    tail_eos = [b for b in range(B) if any(tail[got[b, t]] and got[b, t + 1] == EOS for t in range(steps - 1)
                                           if got[b, t] >= 3)]
    assert tail_eos, "no row ended with a tail token (the grammar would be untested)"
    pick = sorted(set(tail_eos[:6]) | {0, 511, 512, B - 1})
    bias = np.zeros(343, np.float32)
    bias[[0, 1]] = -np.inf
    ref, margin = port.generate(_rows(frames, lens, pick), [2048] * len(pick), steps, bias, 64, return_margin=True)
    # after a row's EOS every token is PAD whatever the logits: margins there do not limit the comparison
    ends = [int(np.argmax(r == EOS)) + 1 if (r == EOS).any() else steps for r in ref]
    ok, identical, stops = _compare(got[pick], ref, margin, caps=ends)
    _report("config 4", ok, identical, stops, steps)
    print(f"config 4: {len(tail_eos)} / {B} rows end with a tail token followed by EOS")
    assert ok.all(), f"rows {np.array(pick)[~ok]} disagree before a low-margin step"


def test_config4_long_horizon_sampled_rows():
    """Config 4 with every row decoding all 280 steps: tails and EOS masked through the bias (the tail rule then
    never fires), and the head's weights scaled by 16.  Scaling the head scales the logits' bf16 errors as much as
    their margins, so the margin floor is scaled with it (16 x 0.05): the comparison is as strict as the plain
    one, over rows that keep decoding to the end (with the untrained 343-way head, near-ties limit how far a row
    can be compared, whatever the scale)."""
    from viktor_b200 import Basecaller, DecodeEngine, DecoderConfig
    from viktor_b200.config import KmerTokenizer
    from viktor_b200.synthetic import make_weights
    B, steps, V = 1024, 280, 343
    cfg = DecoderConfig(vocab_size=V, rope_theta=1e6)
    weights = make_weights(cfg, seed=28, init="torch")
    weights["decoder.lm_head.weight"] = weights["decoder.lm_head.weight"] * 16
    port = TorchCPUModel(OracleConfig(vocab_size=V, rope_theta=1e6), weights, k=4)
    model = Basecaller.from_weights(weights, k=4, cfg=cfg)
    lens = [2048] * B
    frames = _frames(lens, seed=29)
    tail = np.asarray(KmerTokenizer(4).tail_mask, dtype=bool)
    bias = np.zeros(V, np.float32)
    bias[[0, 1, 2]] = -np.inf
    bias[tail] = -np.inf
    eng = DecodeEngine(model, B, steps, 2048, max_homopolymer=None, device="cuda")
    eng.bias.copy_(torch.from_numpy(bias))
    got = eng.generate(frames, lens, steps).cpu().numpy()
    assert (got >= 3).all() and not tail[got].any()
    pick = [0, 255, 256, 511, 512, 767, 900, B - 1]
    ref, margin = port.generate(_rows(frames, lens, pick), [2048] * len(pick), steps, bias, None, return_margin=True)
    ok, identical, stops = _compare(got[pick], ref, margin / 16.0)
    _report("config 4 (long horizon)", ok, identical, stops, steps)
    assert ok.all(), f"rows {np.array(pick)[~ok]} disagree before a low-margin step"


def test_max_seq_len_prefix_and_decode():
    """The decoder's whole position range: a 3000-frame prefix decoded for 1095 steps fills a cache of exactly
    max_seq_len = 4096 positions (BOS at 3000, the last token at 4095: the last RoPE row and cache position),
    beside a short chunk in the same batch.  Four long rows, so that some of them are compared up to the last
    position (a row stops being compared at its first fp32 near-tie)."""
    from viktor_b200 import DecodeEngine
    steps, lens = 1095, [3000, 3000, 100, 3000, 3000]
    model, port = _model(7, 1, seed=31)
    frames = _frames(lens, seed=32)
    eng = DecodeEngine(model, len(lens), steps, max(lens), max_homopolymer=None, device="cuda")
    assert eng.cache.k.shape[2] == 4096
    eng.bias[EOS] = float("-inf")
    got = eng.generate(frames, lens, steps).cpu().numpy()
    bias = np.zeros(7, np.float32)
    bias[[0, 1, 2]] = -np.inf
    ref, margin = port.generate(_rows(frames, lens, range(len(lens))), lens, steps, bias, None,
                                return_margin=True)
    ok, identical, stops = _compare(got, ref, margin)
    _report("max_seq_len", ok, identical, stops, steps)
    print("max_seq_len: steps compared per row", stops.tolist())
    assert ok.all(), f"rows {np.arange(len(lens))[~ok]} disagree before a low-margin step"


def test_config6_2048_chunk_engine_batch():
    """Configs 5 and 6 decode 2048 chunks in one engine batch: 16 prefill sub-batches of 128 and two decode
    groups of 1024 rows.  Config-3 lengths and per-chunk decode lengths (round(128 x frames / 2048), then EOS);
    sampled: the shortest and longest chunks, sub-batch boundaries and the rows either side of the group
    boundary."""
    from viktor_b200 import DecodeEngine
    from viktor_b200.synthetic import varlen_prefix_lengths
    B, steps = 2048, 128
    model, port = _model(7, 1, seed=33)
    lens = varlen_prefix_lengths(B, seed=34)
    caps = [int(round(steps * n / 2048)) for n in lens]
    frames = _frames(lens, seed=35)
    eng = DecodeEngine(model, B, steps, 2048, prefill_batch=128, max_homopolymer=None, device="cuda")
    eng.bias[EOS] = float("-inf")
    eng.max_tokens.copy_(torch.tensor(caps))
    got = eng.generate(frames, lens, None).cpu().numpy()
    pick = sorted({int(np.argmin(lens)), int(np.argmax(lens)), 0, 127, 128, 895, 1023, 1024, 1025, 1920, B - 1})
    bias = np.zeros(7, np.float32)
    bias[[0, 1, 2]] = -np.inf
    ref, margin = port.generate(_rows(frames, lens, pick), [lens[r] for r in pick], steps, bias, None,
                                return_margin=True)
    pc = [caps[r] for r in pick]
    for i, c in enumerate(pc):  # the cap: EOS in column c, PAD after
        if c < steps:
            ref[i, c] = EOS
            ref[i, c + 1:] = PAD
    ok, identical, stops = _compare(got[pick], ref, margin, caps=pc)
    _report("config 6 batch", ok, identical, stops, steps)
    assert ok.all(), f"rows {np.array(pick)[~ok]} disagree before a low-margin step"
    for b in range(B):  # every row: bases up to its cap, then EOS and PAD
        c = caps[b]
        assert (got[b, :min(c, steps)] >= 3).all()
        if c < steps:
            assert got[b, c] == EOS and (got[b, c + 1:] == PAD).all()


def test_config2_full_size_int8_prefix():
    """The opt-in int8 prefix mode at config 2 size (256 x 2048 frames, 256 steps, both decode groups): the
    sampled rows agree with the fp32 port up to their first step whose top-2 margin is below 0.1, the mode's
    own floor (twice the bf16 path's: the quantisation noise of the prefix)."""
    from viktor_b200 import DecodeEngine
    B, steps, floor = 256, 256, 0.1
    model, port = _model(7, 1, seed=21)
    lens = [2048] * B
    frames = _frames(lens, seed=22)
    eng = DecodeEngine(model, B, steps, 2048, max_homopolymer=None, device="cuda", kv_int8=True)
    eng.bias[EOS] = float("-inf")
    got = eng.generate(frames, lens, steps).cpu().numpy()
    pick = list(range(3, B, 17))[:15]
    bias = np.zeros(7, np.float32)
    bias[[0, 1, 2]] = -np.inf
    ref, margin = port.generate(_rows(frames, lens, pick), [2048] * len(pick), steps, bias, None, return_margin=True)
    stops = []
    for i in range(len(pick)):
        low = np.where(np.nan_to_num(margin[i], nan=np.inf) < floor)[0]
        stops.append(int(low[0]) if len(low) else steps)
    ok = np.array([np.array_equal(got[r, :s], ref[i, :s]) for i, (r, s) in enumerate(zip(pick, stops))])
    identical = (got[pick] == ref).all(1)
    _report("config 2 int8 prefix", ok, identical, np.array(stops), steps)
    assert ok.all(), f"rows {np.array(pick)[~ok]} disagree before a step of margin < {floor}"
