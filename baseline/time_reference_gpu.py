"""Times the reference's own paths next to this package's, for context (not the bench contract).

The reference (GHSSHG/Viktor) is installed, unmodified, into baseline/_ref:

    python -m pip install --no-index --no-build-isolation --find-links /opt/wheelhouse --no-deps \
        --target baseline/_ref <copy of the reference checkout>

and imported from there.  Parts (each prints one JSON line):

  --gpu   on one GPU, BASELINE config 2 shapes (256 chunks x 2048 frames, vocab 7, bf16, N(0, 0.02) weights):
          * the reference DecodeEngine(backend="triton") with attention_backend "flash" (its default off sm80,
            viktor/fast_decoder.py:22-30) and "triton" (viktor/decode_attention.py): prefill of the batch, and
            the CUDA-graph decode step at prefix 2048 (graph replays timed with CUDA events); a path that does
            not run on this GPU is reported with its error;
          * one layer of decode attention at the run's mean length (2600) for all 256 rows: the reference's
            Triton kernel, flash_attn_with_kvcache as the reference calls it (num_splits=1, identity
            cache_batch_idx) and this package's vk_decode_attention, CUDA events, GB/s of K/V read;
          * this package's DecodeEngine on the same model and inputs (prefill, decode step).
  --cpu   on the host cores: the stock reference DecodeEngine(backend="torch") (fp32) against oracle/decoder_torch.py
          (the port bench.py's reference arm times) on the same sample, decoded bases/s of each.

    python baseline/time_reference_gpu.py --gpu
    python baseline/time_reference_gpu.py --cpu [--cpu-steps 32]
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(HERE, "_ref"))

PLEN, B, STEPS = 2048, 256, 1100


def reference_model(V, k, device, dtype):
    import torch
    from viktor import Basecaller, DecoderConfig, KmerTokenizer
    from viktor_b200.config import DecoderConfig as OurConfig
    from viktor_b200.synthetic import make_weights
    tok = KmerTokenizer(k)
    model = Basecaller(types.SimpleNamespace(d_model=512), tok, DecoderConfig(vocab_size=V, rope_theta=1e6))
    w = make_weights(OurConfig(vocab_size=V, rope_theta=1e6), seed=0, init="normal")
    model.load_state_dict({n: torch.from_numpy(a) for n, a in w.items()}, strict=True)
    model.projector.to(device, dtype)
    model.decoder.to(device, dtype)
    return model.eval(), w


def cuda_time(fn, reps, torch):
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / 1e3 / reps


def gpu_part():
    import torch
    from viktor import DecodeEngine as RefEngine
    dev = torch.device("cuda")
    res = {"gpu": torch.cuda.get_device_name(), "config": "256 chunks x 2048 frames, vocab 7, bf16"}
    model, weights = reference_model(7, 1, dev, torch.bfloat16)
    g = torch.Generator(device=dev)
    g.manual_seed(1)
    lens = [PLEN] * B
    frames = torch.randn(B * PLEN, 512, generator=g, device=dev).to(torch.bfloat16)

    def set_state(eng, p):
        """Decode state of every row at prefix p (what prefill leaves), for timing the step graph alone."""
        eng.plen.fill_(p)
        eng.pos.fill_(p + 1)
        eng.pos32.fill_(p + 1)
        eng.seqlens.fill_(p + 2)
        eng.rpos32.fill_(p + 1)
        eng.tok.fill_(3)
        if hasattr(eng, "step_idx"):
            eng.step_idx.fill_(1)

    for attn in ("flash", "triton"):
        r = {}
        try:
            eng = RefEngine(model, B, STEPS, PLEN, backend="triton", attention_backend=attn)
            eng.bias[2] = float("-inf")
            try:
                r["prefill_ms_per_chunk"] = cuda_time(lambda: eng.prefill(frames, lens), 2, torch) / B * 1e3
            except Exception as e:  # noqa: BLE001 - report what the reference raises on this GPU
                r["prefill_error"] = f"{type(e).__name__}: {str(e).splitlines()[0][:200]}"
            set_state(eng, PLEN)
            n = 100
            r["decode_us_per_step_at_prefix_2048"] = cuda_time(lambda: [eng.graph.replay() for _ in range(n)], 1,
                                                               torch) / n * 1e6
        except Exception as e:  # noqa: BLE001
            r["error"] = f"{type(e).__name__}: {str(e).splitlines()[0][:200]}"
        res[f"reference_triton_engine_attention_{attn}"] = r
        torch.cuda.empty_cache()

    # one layer of decode attention at the mean length of the config-2 run, all 256 rows
    from viktor_b200._lib import call, load
    S = PLEN + 1 + STEPS
    L = PLEN + 1 + STEPS // 2
    k = torch.randn(B, S, 2, 64, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(B, S, 2, 64, generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn(B, 8, 64, generator=g, device=dev).to(torch.bfloat16)
    lengths = torch.full((B,), L, dtype=torch.int32, device=dev)
    nbytes = B * L * 512
    att = {"rows": B, "length": L, "kv_bytes": nbytes}
    try:
        from viktor.decode_attention import decode_attention
        t = cuda_time(lambda: decode_attention(q, k, v, lengths), 20, torch)
        att["reference_triton_us"], att["reference_triton_gbs"] = t * 1e6, nbytes / t / 1e9
    except Exception as e:  # noqa: BLE001
        att["reference_triton_error"] = f"{type(e).__name__}: {str(e).splitlines()[0][:200]}"
    try:
        from flash_attn import flash_attn_with_kvcache
        seq = torch.arange(B, dtype=torch.int32, device=dev)
        t = cuda_time(lambda: flash_attn_with_kvcache(q[:, None], k, v, cache_seqlens=lengths, cache_batch_idx=seq,
                                                      num_splits=1), 20, torch)
        att["flash_attn_kvcache_us"], att["flash_attn_kvcache_gbs"] = t * 1e6, nbytes / t / 1e9
    except Exception as e:  # noqa: BLE001
        att["flash_attn_kvcache_error"] = f"{type(e).__name__}: {str(e).splitlines()[0][:200]}"
    out = torch.empty_like(q)
    ws = torch.zeros(load().vk_decode_attention_workspace_bytes(B, S), dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    t = cuda_time(lambda: call("vk_decode_attention", q.data_ptr(), k.data_ptr(), v.data_ptr(), lengths.data_ptr(),
                               out.data_ptr(), B, 0, B, S, k.stride(0), k.stride(1), ws.data_ptr(), ws.numel(), st),
                  20, torch)
    att["viktor_b200_us"], att["viktor_b200_gbs"] = t * 1e6, nbytes / t / 1e9
    res["decode_attention_one_layer"] = att
    del k, v

    # this package's engine on the same model object (the reference's own Basecaller) and inputs
    from viktor_b200 import DecodeEngine
    eng = DecodeEngine(model, B, STEPS, PLEN, max_homopolymer=None, device=dev)
    eng.bias[2] = float("-inf")
    ours = {"prefill_ms_per_chunk": cuda_time(lambda: eng.prefill(frames, lens), 2, torch) / B * 1e3}
    set_state(eng, PLEN)
    n = 100

    def replay():
        for _ in range(n):
            eng.graph.replay()
    ours["decode_us_per_step_at_prefix_2048"] = cuda_time(replay, 1, torch) / n * 1e6
    res["viktor_b200_engine"] = ours
    print(json.dumps(res), flush=True)


def cpu_part(steps):
    import torch
    from oracle import OracleConfig
    from oracle.decoder_torch import TorchCPUModel
    from viktor import DecodeEngine as RefEngine
    from viktor_b200.synthetic import make_frames
    model, weights = reference_model(7, 1, torch.device("cpu"), torch.float32)
    n = 4
    lens = [PLEN] * n
    frames = make_frames(lens, seed=1)
    res = {"threads": torch.get_num_threads(), "sample": f"{n} chunks x {PLEN} frames, prefill + {steps} steps"}
    eng = RefEngine(model, n, steps, PLEN, backend="torch", cuda_graph=False, max_homopolymer=None)
    eng.bias[2] = float("-inf")
    t0 = time.perf_counter()
    with torch.no_grad():
        out_ref = eng.generate(torch.from_numpy(frames), lens, steps).numpy()
    t_ref = time.perf_counter() - t0
    port = TorchCPUModel(OracleConfig(vocab_size=7, rope_theta=1e6), weights, k=1)
    bias = np.zeros(7, np.float32)
    bias[[0, 1, 2]] = -np.inf
    t0 = time.perf_counter()
    out_port = port.generate(frames, lens, steps, bias, None)
    t_port = time.perf_counter() - t0
    bases = n * steps
    res.update(reference_torch_engine_s=t_ref, reference_bases_per_s=bases / t_ref, port_s=t_port,
               port_bases_per_s=bases / t_port, same_tokens=bool(np.array_equal(out_ref, out_port)))
    print(json.dumps(res), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpu", action="store_true")
    ap.add_argument("--cpu", action="store_true")
    ap.add_argument("--cpu-steps", type=int, default=32)
    a = ap.parse_args()
    if a.cpu:
        cpu_part(a.cpu_steps)
    if a.gpu:
        gpu_part()


if __name__ == "__main__":
    main()
