"""Opt-in INT8 prefix KV on the GPU, through the C-ABI, against the CPU restatement in oracle/kv_int8_np.py.

* vk_kv_quantize: bytes and per-channel scales bit-exact (integer/byte work).
* vk_decode_attention_i8: within 0.01 of the fp64 attention over the dequantized prefix (the bf16
  decode-attention bar of tests/gpu_check.py:32-81 of the reference; measured 0.004); against the bf16-exact
  attention, within 0.01 of the quantisation error the oracle itself makes (the mode's own tolerance, as the
  reference's analysis.md:95 asks: 0.04-0.07 on these deliberately harsh inputs, channel scales spread 30x and
  scores of several units; held below 0.1); all as max |error| / max(1, |reference|), since these outputs are
  larger than 1.
"""

import numpy as np
import pytest
import torch

from oracle import kv_int8_np as oracle8

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda") if torch.cuda.is_available() else None
BF = torch.bfloat16


@pytest.fixture(autouse=True)
def _errors_clear():
    from viktor_b200._lib import check_device_errors
    yield
    torch.cuda.synchronize()
    check_device_errors()


def _cache(R, S, seed):
    """bf16 K/V [R, S, 2, 64] with per-channel magnitudes spread over 30x (outlier channels, as QK-normed keys
    and values have), so per-channel scales matter."""
    g = torch.Generator().manual_seed(seed)
    mag = torch.exp(torch.rand(2, 128, generator=g) * 3.4) * 0.1
    k = (torch.randn(R, S, 128, generator=g) * mag[0]).reshape(R, S, 2, 64)
    v = (torch.randn(R, S, 128, generator=g) * mag[1]).reshape(R, S, 2, 64)
    return k.to(BF).to(DEV), v.to(BF).to(DEV)


def test_kv_quantize_bytes_exact():
    from viktor_b200.ops import PrefixKV8, kv_quantize
    R, S, row0 = 9, 1000, 2
    starts = [0, 1, 127, 128, 129, 700, 1000]
    k, v = _cache(R, S, 11)
    pre = PrefixKV8(R, max(starts), DEV)
    assert pre.S8 == 1024
    st = torch.tensor(starts, dtype=torch.int32, device=DEV)
    kv_quantize(k, v, st, pre, row0=row0)
    torch.cuda.synchronize()
    k8, sk, sv = (t.cpu().numpy() for t in (pre.k8, pre.sk, pre.sv))
    v8t = pre.v8t.permute(0, 2, 1, 3).reshape(R, 128, pre.S8).cpu().numpy()  # tiles -> [rows, 128, S8]
    kf = k.float().cpu().numpy().reshape(R, S, 128)
    vf = v.float().cpu().numpy().reshape(R, S, 128)
    for i, s in enumerate(starts):
        r = row0 + i
        ku, ks = oracle8.quantize_prefix(kf[r, :s])
        vu, vs = oracle8.quantize_prefix(vf[r, :s])
        assert np.array_equal(k8[r, :s], ku), f"K bytes row {r}"
        assert np.array_equal(v8t[r, :, :s], vu.T), f"V bytes row {r}"
        assert np.array_equal(sk[r], ks) and np.array_equal(sv[r], vs), f"scales row {r}"
        pad = -(-s // 128) * 128
        assert (v8t[r, :, s:pad] == 128).all(), "V tile tail holds the byte for 0"
    assert (k8[:row0] == 0).all() and (k8[row0 + len(starts):] == 0).all(), "rows outside the call untouched"


@pytest.mark.parametrize("B,S,tail", [(40, 3200, 1200), (160, 2600, 520)])
def test_decode_attention_i8(B, S, tail):
    from viktor_b200.ops import PrefixKV8, decode_attention_i8, kv_quantize
    g = torch.Generator().manual_seed(B)
    row0 = 3
    k, v = _cache(B + 5, S, B)
    plen = torch.randint(0, S - tail + 1, (B,), generator=g)
    plen[:6] = torch.tensor([0, 1, 128, 129, 2048, S - tail])
    extra = torch.randint(1, tail + 1, (B,), generator=g)
    extra[:3] = torch.tensor([1, tail, 64])
    starts = plen.int().to(DEV)
    lens = (plen + extra).int().to(DEV)
    q = (torch.randn(B, 8, 64, generator=g) * 2).to(BF).to(DEV)
    pre = PrefixKV8(B + 5, int(plen.max()), DEV)
    kv_quantize(k, v, starts, pre, row0=row0)
    # The prefix positions of the bf16 cache are never read again: NaN there must not reach the output.
    pos = torch.arange(S, device=DEV)
    hide = pos[None] < starts[:, None].long()
    kn, vn = k.clone(), v.clone()
    kn[row0:row0 + B][hide] = float("nan")
    vn[row0:row0 + B][hide] = float("nan")
    for _ in range(2):  # the second call reuses the tickets the first one returned to zero
        out = decode_attention_i8(q, kn, vn, pre, starts, lens, tail, row0=row0)
        torch.cuda.synchronize()
        assert torch.isfinite(out).all()
    got = out.float().cpu().numpy()
    qf, kf, vf = (t.float().cpu().numpy() for t in (q, k, v))
    err_oracle = err_bf16 = err_quant = 0.0
    for b in range(B):
        r, L, s = row0 + b, int(lens[b]), int(starts[b])
        ref, *_ = oracle8.decode_attention_i8(qf[b], kf[r, :L], vf[r, :L], s)
        exact = oracle8.decode_attention(qf[b], kf[r, :L], vf[r, :L])
        # errors relative to max(1, |reference|): outputs reach |o| ~ 8 here (channel scales up to 3), where
        # the bf16 rounding of the output alone is 2^-9 |o|
        rel = np.maximum(1.0, np.abs(exact))
        err_oracle = max(err_oracle, float((np.abs(got[b] - ref) / np.maximum(1.0, np.abs(ref))).max()))
        err_bf16 = max(err_bf16, float((np.abs(got[b] - exact) / rel).max()))
        err_quant = max(err_quant, float((np.abs(ref - exact) / rel).max()))
    print(f"max |out - oracle| / max(1, |oracle|) {err_oracle:.5f}; vs bf16 attention {err_bf16:.5f} "
          f"(the oracle's own quantisation error {err_quant:.5f})")
    assert err_oracle < 0.01, f"max |out - oracle| / max(1, |oracle|) = {err_oracle}"
    assert err_bf16 <= err_quant + 0.01, f"max |out - bf16| / max(1, |bf16|) = {err_bf16}, quantisation {err_quant}"
    assert err_quant < 0.1


def test_decode_attention_i8_rejects_bad_ranges():
    """A start at or past the length, or a tail longer than max_tail, sets the device error flag (the query is
    skipped, nothing faults)."""
    from viktor_b200._lib import check_device_errors
    from viktor_b200.ops import PrefixKV8, decode_attention_i8, kv_quantize
    k, v = _cache(4, 512, 5)
    pre = PrefixKV8(4, 256, DEV)
    kv_quantize(k, v, torch.tensor([200, 200, 200, 200], dtype=torch.int32, device=DEV), pre)
    q = torch.randn(4, 8, 64, device=DEV).to(BF)
    for starts, lens in (([200, 200, 200, 200], [200, 300, 300, 300]), ([200] * 4, [300, 300, 300, 500])):
        decode_attention_i8(q, k, v, pre, torch.tensor(starts, dtype=torch.int32, device=DEV),
                            torch.tensor(lens, dtype=torch.int32, device=DEV), 128)
        torch.cuda.synchronize()
        with pytest.raises(RuntimeError, match="kernel error"):
            check_device_errors()


def _agree_until_low_margin(got, ref, margin, floor):
    ok = []
    for b in range(ref.shape[0]):
        low = np.where(np.nan_to_num(margin[b], nan=np.inf) < floor)[0]
        stop = int(low[0]) if len(low) else ref.shape[1]
        ok.append(np.array_equal(got[b, :stop], ref[b, :stop]))
    return np.array(ok)


def test_engine_int8_prefix_tokens():
    """The engine with kv_int8=True on 128 chunks of 64..512 frames, 32 greedy steps, two decode groups, prefill
    in sub-batches: tokens against the fp32 oracle.  Every chunk agrees up to its first step whose fp32 top-2
    margin is below 0.1 (twice the bf16 floor of the bf16 path: the quantisation noise of the prefix), and
    the fraction of chunks identical over all steps is held above 0.9 (bf16 path: 0.969)."""
    from oracle import OracleConfig, OracleModel
    from viktor_b200 import Basecaller, DecodeEngine, DecoderConfig
    from viktor_b200.synthetic import make_frames, make_weights
    cfg = DecoderConfig(vocab_size=7, rope_theta=1e6)
    weights = make_weights(cfg, seed=31, init="torch")
    rng = np.random.default_rng(32)
    lens = [int(v) for v in rng.integers(64, 513, 128)]
    lens[5] = 0  # a chunk with no frames: its prefix is BOS alone
    frames = make_frames(lens, seed=33)
    steps = 32
    model = Basecaller.from_weights(weights, k=1, cfg=cfg)
    outs = {}
    for int8, graph in ((False, True), (True, True), (True, False)):
        eng = DecodeEngine(model, len(lens), steps, max(lens), max_homopolymer=None, device="cuda", kv_int8=int8,
                           prefill_batch=48, cuda_graph=graph)
        eng.bias[2] = float("-inf")
        outs[int8, graph] = eng.generate(torch.from_numpy(frames), lens, steps).cpu().numpy().copy()
        eng.check_errors()
    got = outs[True, True]
    assert np.array_equal(got, outs[True, False]), "graph replay == eager under kv_int8"
    bias = np.zeros(7, np.float32)
    bias[[0, 1, 2]] = -np.inf
    om = OracleModel(OracleConfig(vocab_size=7, rope_theta=1e6), weights, k=1)
    ref, margin = om.generate(frames, lens, steps, steps=steps, bias=bias, max_homopolymer=None)
    ok = _agree_until_low_margin(got, ref, margin, 0.1)
    exact = (got == ref).all(1).mean()
    same_bf16 = (got == outs[False, True]).all(1).mean()
    print(f"kv_int8: identical chunks vs oracle {exact:.4f}, vs bf16 engine {same_bf16:.4f}, "
          f"agree-until-margin {ok.mean():.4f}")
    assert ok.all(), np.where(~ok)[0]
    assert exact >= 0.9


@pytest.mark.parametrize("name", ["base_theta1e6", "base_theta1e4", "kmer4", "homopolymer", "pos_scale2", "base_b8"])
def test_engine_int8_prefix_golden_cases(name):
    """kv_int8=True on the golden cases (4-mer vocabulary and its tail rule, homopolymer stop, pos_scale 2, ragged
    batch of 8): the reference's greedy tokens, up to each row's first step whose fp32 top-2 margin is below 0.1
    (the int8 mode's floor)."""
    from golden_io import load
    from oracle import OracleConfig, OracleModel
    from viktor_b200 import Basecaller, DecodeEngine, DecoderConfig
    g = load(name)
    m = g["meta"]
    model = Basecaller.from_weights(g["weights"], k=m["k"], cfg=DecoderConfig(**m["cfg"]), d_enc=m["d_enc"],
                                    pos_scale=m["pos_scale"])
    eng = DecodeEngine(model, len(m["lens"]), m["max_new"], max(m["lens"]), max_homopolymer=m["max_homopolymer"],
                       device="cuda", kv_int8=True)
    eng.bias.copy_(torch.from_numpy(g["bias"]))
    got = eng.generate(torch.from_numpy(g["frames"]), m["lens"], m["max_new"]).cpu().numpy()
    eng.check_errors()
    om = OracleModel(OracleConfig(**m["cfg"]), g["weights"], k=m["k"], pos_scale=m["pos_scale"])
    _, margin = om.generate(g["frames"], m["lens"], m["max_new"], steps=m["max_new"], bias=g["bias"],
                            max_homopolymer=m["max_homopolymer"])
    ok = _agree_until_low_margin(got, g["tokens"], margin, 0.1)
    print(f"{name}: kv_int8 identical rows {(got == g['tokens']).all(1).mean():.3f}")
    assert ok.all(), f"rows disagreeing before a low-margin step: {np.where(~ok)[0]}"
