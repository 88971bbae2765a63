"""Benchmark of the Viktor decoder hot path on B200: decoded bases/s and microseconds per decode step.

One bench step = one ``DecodeEngine.generate`` per engine batch of this GPU's chunks (packed prefill of the
projected frames, then greedy CUDA-graph decode steps with EOS masked, so every step emits one token per chunk
until the chunk's own decode length).  Default workload: 256 chunks x 2048 frames x
512 features ~ N(0, 1), 1100 decode steps, single-base vocabulary (7), 8-layer d512 GQA 8/2 decoder with
N(0, 0.02) random weights, bf16.  Other BASELINE configs:

    --config 3   512 chunks of U{128..2048 step 128} frames; chunk b decodes round(1100 x frames_b / 2048)
                 tokens, then EOS and PAD (engine.max_tokens); decode(steps=None) stops when every chunk ended
    --config 4   1024 chunks x 2048 frames, 4-mer vocabulary (343), 280 steps
    --config 5   2048 chunks per GPU (config-2 lengths) in one engine batch of 2048 (--engine-batch 256: eight
                 batches of config 2's size), all ranks' tokens gathered to rank 0's host
    --config 6   config 5 with the config-3 workload (varlen prefixes, per-chunk decode lengths)

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 2|3|4|5|6]

Multi-GPU: one process per GPU under torch.distributed.run; every rank runs its own engine on its own chunks
(weak scaling, no collective on the data path); the barrier / max-over-ranks timing uses NCCL, and in the e2e
region the token arrays of all ranks are gathered to rank 0 (NCCL) and copied to its host.

Printed keys beyond the base contract:
  roofline      decode attention (the dominant kernel): algorithmic KV bytes per launch / measured launch time
  cpu_baseline  the reference path on the host cores (PyTorch CPU fp32 port) on a bounded sample, rank 0, N=1
  e2e           the same metric through the public API from pinned host frames, tokens back on one host
  decode_us_per_step (decode_ms_per_batch with per-chunk lengths), prefill_ms_per_chunk, gpu_launches, clocks
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    2: dict(name="config2: 256 chunks x 2048 frames, 1100 greedy steps, vocab 7", B=256, frames="full", steps=1100,
            k=1),
    3: dict(name="config3: 512 chunks x U{128..2048 step 128} frames, decode length 1100 x frames / 2048 (then "
                 "EOS, PAD), vocab 7", B=512, frames="varlen", steps=1100, k=1, budget=True),
    4: dict(name="config4: 1024 chunks x 2048 frames, 280 greedy steps, 4-mer vocab 343", B=1024, frames="full",
            steps=280, k=4),
    5: dict(name="config5: 2048 chunks per GPU x 2048 frames (config-2 lengths), 1100 greedy steps, vocab 7, "
                 "tokens of every rank gathered to rank 0's host", B=2048, engine_batch=2048, frames="full",
            steps=1100, k=1),
    # config 5 with the config-3 workload (varlen prefixes, per-chunk decode lengths) at 2048 chunks per GPU
    6: dict(name="config5 with config-3 lengths: 2048 chunks per GPU x U{128..2048 step 128} frames, decode "
                 "length 1100 x frames / 2048 (then EOS, PAD), vocab 7, tokens of every rank gathered to rank 0's "
                 "host", B=2048, engine_batch=2048, frames="varlen", steps=1100, k=1, budget=True),
}
PLEN = 2048
HBM_FALLBACK_GBS = 6650.0


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    return HBM_FALLBACK_GBS, "fallback"


def ncu_traffic_ratio():
    """DRAM bytes / algorithmic bytes of one decode-attention launch, from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "decode_attention_config2.md")
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.startswith("traffic_over_algorithmic:"):
            return float(line.split(":")[1])
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples taken while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def make_lens(cfg, B, seed):
    from viktor_b200.synthetic import varlen_prefix_lengths
    return [PLEN] * B if cfg["frames"] == "full" else varlen_prefix_lengths(B, seed=seed)


def make_budgets(cfg, lens):
    """Per-chunk decode lengths of the workload: with cfg["budget"] (config 3), round(steps x frames / 2048)
    tokens and then EOS; otherwise None (every chunk decodes the full number of steps, EOS masked)."""
    if not cfg.get("budget"):
        return None
    return [int(round(cfg["steps"] * n / PLEN)) for n in lens]


def cpu_baseline(args, cfg, steps=None):
    """The reference path on the host cores: a multithreaded PyTorch-CPU fp32 restatement (oracle/decoder_torch.py,
    pinned to the reference's golden tokens) on a bounded sample of the same workload: 4 chunks (2048 frames, or
    the varlen workload's lengths), prefill + the workload's number of greedy steps (or `steps`).  With per-chunk
    decode lengths the batch runs until its longest chunk is done, as the reference engine does (finished rows
    keep computing PAD), and only the bases each chunk emits before its end are counted."""
    import torch
    from oracle import OracleConfig
    from oracle.decoder_torch import TorchCPUModel
    from viktor_b200.config import DecoderConfig
    from viktor_b200.synthetic import make_frames, make_weights
    B = 4
    steps = steps or args.cpu_steps or cfg["steps"]
    V = 7 if cfg["k"] == 1 else 343
    dc = DecoderConfig(vocab_size=V, rope_theta=1e6)
    tm = TorchCPUModel(OracleConfig(vocab_size=V, rope_theta=1e6), make_weights(dc, seed=0, init="normal"),
                       k=cfg["k"])
    lens = make_lens(cfg, B, seed=7)
    budgets = make_budgets(dict(cfg, steps=steps), lens)
    run_steps = steps if budgets is None else max(budgets) + 1
    frames = make_frames(lens, seed=1)
    bias = np.zeros(V, np.float32)
    bias[[0, 1, 2]] = -np.inf
    t0 = time.perf_counter()
    out = tm.generate(frames, lens, run_steps, bias, None)
    dt = time.perf_counter() - t0
    nb = tm.tok.n_bases[out]
    if budgets is not None:
        nb = nb * (np.arange(out.shape[1])[None, :] < np.asarray(budgets)[:, None])
    bases = int(nb.sum())
    what = f"{PLEN} frames" if cfg["frames"] == "full" else f"frames {lens}, decode lengths {budgets}"
    return {"value": bases / dt, "unit": "bases/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{B} chunks x {what}, prefill + {run_steps} greedy steps, PyTorch CPU fp32 restatement "
                      f"of the reference path ({dt:.1f} s)", "seconds": dt}


def run_reference_arm(args, cfg, rank):
    if rank != 0:
        return
    for _ in range(args.warmup):  # untimed warm-up steps on a short sample (the same code path, 16 decode steps)
        cpu_baseline(args, cfg, steps=16)
    res = [cpu_baseline(args, cfg) for _ in range(max(1, args.steps))]
    vals = [r["value"] for r in res]
    v = statistics.median(vals)
    ms = statistics.median(r.pop("seconds") for r in res) * 1e3
    line = {"metric": "decoded bases/s", "value": v, "unit": "bases/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": cfg["name"], "sample": res[0]["sample"]},
            "cpu_baseline": dict(res[0], value=v),
            "e2e": {"value": v, "unit": "bases/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def attention_roofline(eng, torch, mids):
    """Average launch time of the decode attention kernel with each row at its mean decode length of the run
    (mids: prefix + 1 + half the row's decode length), timed with CUDA events on the launching stream;
    algorithmic bytes = K and V rows read + q read + o written."""
    from viktor_b200._lib import call
    B = eng.B
    mid = torch.tensor(mids, dtype=torch.int32, device=eng.device)
    st = torch.cuda.current_stream(eng.device)
    reps = 5
    kc, vc = eng.cache.k, eng.cache.v

    def launch(i):
        call("vk_decode_attention", eng.q.data_ptr(), kc[i].data_ptr(), vc[i].data_ptr(), mid.data_ptr(),
             eng.o.data_ptr(), B, 0, kc.shape[1], kc.shape[2], kc[i].stride(0), kc[i].stride(1),
             eng.attn_ws.data_ptr(), eng.attn_ws.numel(), st.cuda_stream)

    for i in range(8):
        launch(i)
    torch.cuda.synchronize(eng.device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        for i in range(8):
            launch(i)
    e1.record(st)
    torch.cuda.synchronize(eng.device)
    t = e0.elapsed_time(e1) / 1e3 / (reps * 8)
    nbytes = int(mid.long().sum().item()) * 512 + B * 1024 * 2
    return nbytes, t


def attention_roofline_i8(eng, torch, mids):
    """The same measurement for the opt-in int8-prefix kernel (vk_decode_attention_i8): algorithmic bytes =
    int8 prefix (256 B per position) + bf16 tail (512 B per position) + per-channel scales + q read + o written."""
    from viktor_b200._lib import call
    B = eng.B
    mid = torch.tensor(mids, dtype=torch.int32, device=eng.device)
    st = torch.cuda.current_stream(eng.device)
    reps = 5
    kc, vc = eng.cache.k, eng.cache.v
    from viktor_b200._lib import load
    ws = torch.zeros(load().vk_decode_attention_i8_workspace_bytes(B, eng.prefix8[0].S8, eng.max_tail),
                     dtype=torch.uint8, device=eng.device)

    def launch(i):
        pre = eng.prefix8[i]
        call("vk_decode_attention_i8", eng.q.data_ptr(), kc[i].data_ptr(), vc[i].data_ptr(), pre.k8.data_ptr(),
             pre.v8t.data_ptr(), pre.sk.data_ptr(), pre.sv.data_ptr(), eng.starts.data_ptr(), mid.data_ptr(),
             eng.o.data_ptr(), B, 0, kc.shape[1], kc.shape[2], kc[i].stride(0), kc[i].stride(1), pre.S8,
             eng.max_tail, ws.data_ptr(), ws.numel(), st.cuda_stream)

    for i in range(8):
        launch(i)
    torch.cuda.synchronize(eng.device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        for i in range(8):
            launch(i)
    e1.record(st)
    torch.cuda.synchronize(eng.device)
    t = e0.elapsed_time(e1) / 1e3 / (reps * 8)
    starts = eng.starts.long()
    nbytes = int(starts.sum().item()) * 256 + int((mid.long() - starts).sum().item()) * 512 + B * (1024 * 2 + 1024)
    return nbytes, t


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, choices=sorted(CONFIGS), default=2)
    ap.add_argument("--decode-steps", type=int, default=None, help="override the workload's decode steps")
    ap.add_argument("--batch", type=int, default=None, help="override the workload's chunks per GPU (profiling)")
    ap.add_argument("--engine-batch", type=int, default=None,
                    help="chunks per DecodeEngine batch (default: the workload's; config 5: 2048)")
    ap.add_argument("--decode-groups", type=int, default=2, help="row groups decoded on concurrent streams")
    ap.add_argument("--cpu-steps", type=int, default=None, help="CPU-baseline decode steps (default: workload's)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--kv-int8", action="store_true",
                    help="opt-in int8 prefix KV (own tolerance; the headline number is the bf16 path)")
    args = ap.parse_args()
    cfg = dict(CONFIGS[args.config])
    if args.decode_steps:
        cfg["steps"] = args.decode_steps
    if args.batch:
        cfg["B"] = args.batch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference_arm(args, cfg, rank)
        return

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)

    from viktor_b200 import Basecaller, DecodeEngine, DecoderConfig
    from viktor_b200 import _lib
    from viktor_b200.synthetic import make_weights

    B_total, steps = cfg["B"], cfg["steps"]
    eb = args.engine_batch or cfg.get("engine_batch", B_total)
    if B_total % eb:
        raise SystemExit(f"--engine-batch {eb} must divide the {B_total} chunks per GPU")
    nbat = B_total // eb
    V = 7 if cfg["k"] == 1 else 343
    dcfg = DecoderConfig(vocab_size=V, rope_theta=1e6)
    model = Basecaller.from_weights(make_weights(dcfg, seed=0, init="normal"), k=cfg["k"], cfg=dcfg)
    lens_all = make_lens(cfg, B_total, seed=100 + rank)
    budgets_all = make_budgets(cfg, lens_all)
    eng = DecodeEngine(model, eb, steps, PLEN, max_homopolymer=None, device=dev, decode_groups=args.decode_groups,
                       kv_int8=args.kv_int8)
    eng.bias[2] = float("-inf")  # EOS masked: every step emits a base until a chunk's own decode length
    decode_arg = None if budgets_all is not None else steps  # per-chunk lengths: stop when every chunk ended
    n_bases = torch.as_tensor(model.tokenizer.n_bases, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(1 + rank)
    frames = torch.randn(sum(lens_all), 512, generator=g, device=dev)
    offs = np.concatenate([[0], np.cumsum(lens_all)]).astype(np.int64)
    batches = []  # (frames, lens, decode lengths on the device or None) of each engine batch of this rank
    for j in range(nbat):
        lo, hi = j * eb, (j + 1) * eb
        bud = None if budgets_all is None else torch.tensor(budgets_all[lo:hi], dtype=torch.long, device=dev)
        batches.append((frames[int(offs[lo]):int(offs[hi])], lens_all[lo:hi], bud))

    def set_budget(bud):
        if bud is not None:
            eng.max_tokens.copy_(bud)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    st = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        for fr, ln, bud in batches:
            set_budget(bud)
            eng.generate(fr, ln, decode_arg)
    eng.check_errors()

    # ---- device-resident timed region ----
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(args.steps * nbat)]
    bases = torch.zeros((), dtype=torch.long, device=dev)
    launches0 = _lib.launches
    barrier()
    with ClockSampler(local) as clk:
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(st)
        for i in range(args.steps):
            for j, (fr, ln, bud) in enumerate(batches):
                e0, e1, e2 = ev[i * nbat + j]
                set_budget(bud)
                e0.record(st)
                eng.prefill(fr, ln)
                e1.record(st)
                out = eng.decode(decode_arg)
                e2.record(st)
                bases += n_bases[out].sum()
        t_end.record(st)
        barrier()
    launches = _lib.launches - launches0
    elapsed = t_start.elapsed_time(t_end) / 1e3
    prefill_s = sum(a.elapsed_time(b) for a, b, _ in ev) / 1e3
    decode_s = sum(b.elapsed_time(c) for _, b, c in ev) / 1e3
    bases_rank = int(bases.item())
    eng.check_errors()
    if world > 1:
        from viktor_b200.parallel import reduce_bench
        elapsed, decode_s, prefill_s, total_bases = reduce_bench(elapsed, decode_s, prefill_s, bases_rank, dev)
    else:
        total_bases = bases_rank
    value = total_bases / elapsed

    # ---- end to end through the public API: pinned host frames in, tokens back to one host ----
    # Every engine batch is generated from pinned host frames (copied per prefill sub-batch inside generate) and
    # its tokens go into this rank's int16 token array on the device; at the end of the step the arrays of all
    # ranks are gathered to rank 0 (NCCL) and copied into its pinned host memory, where the bases are counted.
    # The batches of a shard reuse batch 0's host frames (one pinned engine batch of frames per rank).
    e2e = None
    if not args.no_e2e:
        from viktor_b200.parallel import gather_tokens, reduce_bench
        fr0, ln0, _ = batches[0]
        host_frames = fr0.cpu().pin_memory()
        tok_dev = torch.empty(B_total, steps, dtype=torch.int16, device=dev)
        host_tok = torch.empty(world * B_total, steps, dtype=torch.int16).pin_memory() if rank == 0 else None
        nb_host = np.asarray(model.tokenizer.n_bases)

        def e2e_step():
            for j, (_, _, bud) in enumerate(batches):
                set_budget(bud)
                out = eng.generate(host_frames, ln0, decode_arg)
                tok_dev[j * eb:(j + 1) * eb].copy_(out)
            if world > 1:
                got = gather_tokens(tok_dev, host_out=host_tok)
            else:
                host_tok.copy_(tok_dev, non_blocking=True)
                st.synchronize()
                got = host_tok
            return 0 if got is None else int(nb_host[got.numpy()].sum())

        e2e_step()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        hb = 0
        for _ in range(args.steps):
            hb += e2e_step()
        e1.record(st)
        barrier()
        t_e2e = e0.elapsed_time(e1) / 1e3
        if world > 1:
            t_e2e, _, _, hb = reduce_bench(t_e2e, 0.0, 0.0, hb, dev)
        e2e = {"value": hb / t_e2e, "unit": "bases/s", "h2d_bytes_per_step": nbat * host_frames.numel() * 4,
               "d2h_bytes_per_step": world * B_total * steps * 2,
               "note": "h2d per rank (fp32 frames, every engine batch); d2h = int16 tokens of all ranks into rank "
                       "0's pinned memory" + (" after an NCCL gather" if world > 1 else "")}

    d0 = budgets_all[:eb] if budgets_all is not None else [steps] * eb
    mids = [n + 1 + d // 2 for n, d in zip(batches[0][1], d0)]
    nbytes, t_attn = attention_roofline(eng, torch, mids)
    peak, peak_kind = peaks()
    achieved = nbytes / t_attn / 1e9
    ratio = ncu_traffic_ratio()
    roofline = {"bound": "hbm", "kernel": "decode_attn_kernel", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                if peak_kind == "measured" else "fallback 6.65 TB/s",
                "bytes_per_launch": nbytes, "launch_us": t_attn * 1e6,
                "traffic": None if ratio is None else nbytes * ratio}
    roofline_i8 = None
    if args.kv_int8:
        nb8, t8 = attention_roofline_i8(eng, torch, mids)
        roofline_i8 = {"bound": "hbm", "kernel": "decode_attn_i8_kernel", "achieved": nb8 / t8 / 1e9, "peak": peak,
                       "unit": "GB/s", "frac": nb8 / t8 / 1e9 / peak, "bytes_per_launch": nb8,
                       "launch_us": t8 * 1e6}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args, cfg)
        cpu.pop("seconds")

    if rank == 0:
        n_gen = args.steps * nbat
        line = {"metric": "decoded bases/s", "value": value, "unit": "bases/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": cfg["name"], "global_batch": B_total * world, "engine_batch": eb,
                           "seq_len": PLEN + 1 + steps, "parallelism": f"dp{world} (independent chunk shards)",
                           "l2": "inputs larger than L2 (KV cache 2 x 8 x B x 3149 x 256 B = 3.3 GB per 256 chunks)"},
                "prefill_ms_per_chunk": prefill_s / (n_gen * eb) * 1e3,
                "gpu_launches": launches, "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
                "clocks": clk.summary()}
        if budgets_all is None:
            line["decode_us_per_step"] = decode_s / (n_gen * (steps - 1)) * 1e6
        else:
            line["decode_ms_per_batch"] = decode_s / n_gen * 1e3
            line["config"]["decode_lengths"] = "per chunk round(1100 x frames / 2048) tokens, then EOS (max_tokens)"
        if args.kv_int8:
            line["config"]["kv_int8"] = "prefix K/V int8 with per-channel scales, generated tokens bf16"
            line["roofline_int8"] = roofline_i8
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
