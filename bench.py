#!/usr/bin/env python
"""Benchmark of the B200 IndexTTS-2.5 Stage-1 decoder.

Default workload (N=1): configs[1], batch-1 long-context decode: 32 conditioning
latents + 600 text tokens, then 1500 sampled mel tokens (T 0.8, top-k 30, top-p 0.8,
repetition penalty 10), seeded synthetic weights (N(0, 0.02), int8 g64 affine, fp16
scales/biases).  One step = one generate call (prefill + 1500 decode steps); STOP is
masked (min_codes = 1500) so every step decodes the same 1500 tokens.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Multi-GPU (torchrun, one process per GPU): request-level data parallelism, every rank
decodes its own requests; no collective on the data path (a gloo barrier and a max of
the per-rank times only).  value = mel tokens of all ranks / max-over-ranks time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "index-tts-rs_b200"))

N_CONDS = 32
N_TEXT = 600
N_MEL = 1500
LANG = 1
SAMPLING = dict(top_k=30, top_p=0.8, temperature=0.8, repetition_penalty=10.0)
WORKLOAD = ("cfg2: batch 1, 32 fp16 N(0,1) conds + 600 uniform text tokens, 1500 sampled mel "
            "tokens (T 0.8, top-k 30, top-p 0.8, rep 10; STOP masked so all 1500 decode), "
            "KV grows 635 -> 2134")


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), \
        int(os.environ.get("LOCAL_RANK", 0))


def max_over_ranks(values, world: int):
    """Element-wise max of a vector of times over the ranks (gloo all-reduce); the job's
    time is its slowest rank's."""
    import numpy as _np
    if world <= 1:
        return _np.asarray(values, _np.float64)
    import torch
    import torch.distributed as dist
    t = torch.tensor(_np.asarray(values, _np.float64), dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.numpy()


def job_throughput(units_per_rank: int, world: int, seconds_max: float) -> float:
    """Whole-job units per second: every rank processed units_per_rank (weak scaling),
    timed by the slowest rank."""
    return units_per_rank * world / seconds_max


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except (OSError, ValueError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


METRIC = "mel tokens/s (cfg2 batch-1 decode)"
XK_TRAFFIC = 686_756_096 + 5_795_328  # DRAM bytes of one batch-1 decode-step launch (ncu)
DTYPE = "int8 weights (g64 affine, fp16 scales) x fp16 activations and KV, fp32 accumulate"


def make_model(seed=2024, synth_path=None):
    from itts_gpt.synth import ModelConfig, make_weights
    cfg = ModelConfig()
    return cfg, make_weights(cfg, seed=seed, synth_path=synth_path)


def make_prompt(cfg, rank: int, synth_path=None):
    from itts_gpt.synth import make_conds, make_text
    text = make_text(N_TEXT, cfg.text_vocab, seed=100 + rank)
    conds = make_conds(cfg.d, N_CONDS, seed=200 + rank, synth_path=synth_path)
    return text, conds


def kv_bytes_per_step(cfg, L):
    return cfg.n_layers * 2 * cfg.d * 2 * L  # fp16 K and V over L positions


# KV lengths (positions before the step) at which the CPU decode step is timed: the cfg2
# decode runs steps at 635 .. 2133 cached positions.
CPU_KV_SAMPLES = (635, 1010, 1385, 1760, 2133)


def cpu_baseline(cfg, w, text, conds, threads: int, steps_per_len: int = 2) -> dict:
    """The CPU restatement (oracle/) on a bounded sample of the cfg2 workload, all host
    threads: the full 635-position prefill, then `steps_per_len` sampled decode steps at
    each KV length of CPU_KV_SAMPLES (the cache is extended to that length between
    samples).  A step's cost is linear in its KV length (fixed weight work + attention
    over the cache), so the 1500 steps of cfg2 are integrated from the samples by the
    trapezoid rule over KV lengths 635 .. 2133."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as orc
    om = orc.OracleModel(w, n_threads=threads)
    kv = om.kv(N_CONDS + N_TEXT + 3 + N_MEL)
    t0 = time.perf_counter()
    logits = om.prefill(kv, text, conds, LANG)
    prefill_s = time.perf_counter() - t0
    seen = np.zeros(129, np.uint64)
    orc.lib().orc_seen_initial(seen.ctypes.data)
    params = orc.params_c(False, SAMPLING["top_k"], SAMPLING["top_p"], SAMPLING["temperature"],
                          SAMPLING["repetition_penalty"])
    state = orc.lib().orc_rng_new(7)
    per_len = []
    for L in CPU_KV_SAMPLES:
        if kv.valid_len() < L:
            kv.fill(L)
        ts = []
        for _ in range(steps_per_len):
            logits[8193] = -np.inf
            t1 = time.perf_counter()
            tok, state = orc.sample_next_token(logits, seen, params, state)
            orc.lib().orc_seen_insert(seen.ctypes.data, tok)
            logits = om.step(kv, tok, 2 + kv.valid_len() - (N_CONDS + N_TEXT + 3))
            ts.append(time.perf_counter() - t1)
        per_len.append(min(ts))
    xs = np.array(CPU_KV_SAMPLES, np.float64)
    ys = np.array(per_len, np.float64)
    lens = np.arange(N_CONDS + N_TEXT + 3, N_CONDS + N_TEXT + 3 + N_MEL - 1, dtype=np.float64)
    decode_s = float(np.interp(lens, xs, ys).sum())
    per_token = (prefill_s + decode_s) / N_MEL
    sample_s = prefill_s + sum(steps_per_len * y for y in per_len)
    return {"value": 1.0 / per_token, "unit": "mel tokens/s", "cores": threads, "kind": "port",
            "sample": (f"cfg2 prefill ({N_CONDS + N_TEXT + 3} positions, {prefill_s:.2f} s) + "
                       f"{steps_per_len} sampled decode steps at each KV length "
                       f"{list(CPU_KV_SAMPLES)} ({', '.join(f'{1000 * y:.1f}' for y in per_len)} "
                       f"ms/step); value = 1500 / (prefill + the 1499 steps' cost interpolated "
                       f"linearly between those KV lengths)"),
            "ms_per_mel_token": 1000.0 * per_token, "sample_seconds": sample_s,
            "extrapolated_decode_s": decode_s}


def run_reference(args, rank, world):
    """Reference arm: the reference itself (Rust + MLX/Metal) cannot be built here, so the
    CPU restatement of its algorithm (oracle/) runs on all host threads.  Weights and
    prompt come from the oracle's own build of the seeded generator, so this arm loads no
    library of the product."""
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as orc
    sp = orc.synth_lib_path()
    threads = os.cpu_count() or 1
    cfg, w = make_model(synth_path=sp)
    text, conds = make_prompt(cfg, 0, synth_path=sp)
    vals = []
    for i in range(args.warmup + args.steps):
        r = cpu_baseline(cfg, w, text, conds, threads)
        if i >= args.warmup:
            vals.append(r)
    value = statistics.mean(v["value"] for v in vals)
    sample_ms = 1000.0 * statistics.mean(v["sample_seconds"] for v in vals)
    line = {"impl": "reference", "metric": METRIC, "value": value,
            "unit": "mel tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": sample_ms,
            "ms_per_mel_token": 1000.0 / value, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "parallelism": "host threads",
                       "step": "one bounded CPU sample of cfg2 (prefill + decode steps at 5 KV "
                               "lengths); ms_per_step is that sample's wall time"},
            "cpu_baseline": {"value": value, "unit": "mel tokens/s", "cores": threads,
                             "kind": "port", "sample": vals[0]["sample"]},
            "e2e": {"value": value, "unit": "mel tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "note": "reference is Rust + MLX (Metal); not buildable on this box "
                    "(no cargo/rustc, no MLX); the CPU restatement of its algorithm stands in"}
    print(json.dumps(line), flush=True)


def run_ours(args, rank, world, local_rank):
    import itts_gpt as ig

    peaks = {}
    pp = ROOT / "MEASURED_PEAKS.json"
    if pp.exists():
        peaks = json.loads(pp.read_text())
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"

    cfg, w = make_model()
    gpt = ig.Gpt.from_weights(w, device=local_rank)
    text, conds = make_prompt(cfg, rank)
    max_seq = N_CONDS + N_TEXT + 3 + N_MEL + 40
    kv = ig.KvCache(gpt, max_seq=max_seq, max_batch=1)
    params = ig.SamplingParams(max_mel_tokens=N_MEL, **SAMPLING)
    prompt = ig.CodePrompt(text, conds, LANG, min_codes=N_MEL)

    def one_step(seed):
        return ig.generate_codes_after(gpt, prompt, kv, params, ig.SamplerRng(seed))

    for i in range(args.warmup):
        codes = one_step(i)
        assert len(codes) == N_MEL, len(codes)

    import torch
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    torch.cuda.set_device(local_rank)
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    clocks.start()
    dev_ms, wall = 0.0, 0.0
    launches = 0
    prefill_ms = 0.0
    t0 = time.perf_counter()
    for i in range(args.steps):
        ts = time.perf_counter()
        codes = one_step(1000 + i)
        wall += time.perf_counter() - ts
        pf, dc, nl = gpt.last_timing()
        dev_ms += pf + dc
        prefill_ms += pf
        launches += nl
        assert len(codes) == N_MEL
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()

    # the decode-step forward (one launch), timed alone at the mean KV length
    L_avg = N_CONDS + N_TEXT + 3 + (N_MEL - 1) // 2
    kname = kv.decode_kernel(1)
    kdesc = {"xk_decode_kernel": "decode step on one 6-CTA cluster per attention head (120 CTAs): q/k/v and "
                                 "attention partials stay in the cluster, stage inputs gathered once per cluster "
                                 "(int8 g64 dequant GEMVs + flash-decode attention)",
             "mk_decode_kernel": "persistent grid-wide decode step (int8 g64 dequant GEMVs + flash-decode "
                                 "attention)"}.get(kname, "decode step")
    ws_ms, ws_launches = _bench_decode_forward(gpt, kv, L_avg, iters=100)
    wbytes = cfg.weight_bytes()
    step_bytes = wbytes + kv_bytes_per_step(cfg, L_avg + 1)

    times = max_over_ranks([dev_ms / 1000.0, wall], world)
    dev_s, wall_s = float(times[0]), float(times[1])
    tokens = N_MEL * args.steps * world
    cfg5 = None
    if not args.no_extra:
        kv.close()
        cfg5 = bench_cfg5(cfg, w, rank, world, local_rank)
    if rank != 0:
        return
    # kernels of ours per generate: prefill (embed + 7 per layer + 2 LN + head GEMM),
    # the first sample, then per decode step the forward (ws_launches) + the sampler
    prefill_k = 1 + 7 * cfg.n_layers + 3
    step_k = ws_launches + 1
    gpu_launches = args.steps * (prefill_k + 1 + step_k * (N_MEL - 1))
    h2d = 4 * (N_TEXT + 2) + 4 * N_CONDS * cfg.d
    d2h = 4 * N_MEL
    achieved = step_bytes / (ws_ms * 1e-3) / 1e9
    line = {
        "metric": METRIC,
        "value": job_throughput(N_MEL * args.steps, world, dev_s), "unit": "mel tokens/s",
        "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000.0 * dev_s / args.steps,
        "ms_per_mel_token": 1000.0 * dev_s / (N_MEL * args.steps),
        "prefill_ms_per_request": prefill_ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": DTYPE,
        "data": "synthetic (seeded N(0,0.02) weights, int8 g64 affine, fp16 scales/biases)",
        "config": {"workload": WORKLOAD, "global_batch": world, "seq_len": int(max_seq),
                   "parallelism": f"request replicas x{world} (no collectives)",
                   "l2": "no flush needed: every decode step streams 514 MB of weights (> 126 MB L2)",
                   "weights_bytes_per_step": wbytes,
                   "kv_bytes_per_step_avg": kv_bytes_per_step(cfg, L_avg)},
        "e2e": {"value": job_throughput(N_MEL * args.steps, world, wall_s), "unit": "mel tokens/s",
                "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": int(gpu_launches),
        "roofline": {"bound": "hbm", "kernel": f"{kname} ({kdesc}, one launch per token)",
                     "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "peak_source": peak_src,
                     "algorithmic_bytes_per_launch": step_bytes,
                     "bytes_formula": "514,144,936 weight B + 122,880 B x KV positions (fp16 K+V)",
                     "kv_positions": L_avg + 1, "launches_per_step": ws_launches,
                     "ms_per_launch": ws_ms,
                     # dram__bytes_read.sum + dram__bytes_write.sum of one launch at this KV
                     # length, from an ncu capture of this kernel build (not measured here)
                     "traffic": XK_TRAFFIC if kname == "xk_decode_kernel" else None,
                     "traffic_source": "ncu --set full capture of one xk_decode_kernel launch at KV 1,384 "
                                       "(686,756,096 B read + 5,795,328 B written); not measured in this run"},
        "clocks": clk,
    }
    if cfg5 is not None:
        line["cfg5"] = cfg5
    if world == 1 and not args.no_extra:
        for key, fn in (("codec_decode", lambda: bench_codec(codes)),
                        ("cfg1", lambda: bench_cfg1(cfg, gpt, w)),
                        ("prefill_cfg4", lambda: bench_prefill_cfg4(cfg, gpt, peaks)),
                        ("cfg3", lambda: bench_cfg3(cfg, gpt, peaks))):
            try:
                line[key] = fn()
            except Exception as e:  # never blocks the headline line
                line[key] = {"error": str(e)[:300]}
    if not args.no_cpu_baseline:
        try:
            line["cpu_baseline"] = cpu_baseline(cfg, w, text, conds, os.cpu_count() or 1)
        except Exception as e:  # the baseline never blocks the GPU line
            line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    print(json.dumps(line), flush=True)


def bench_codec(codes) -> dict:
    """The step after the decoder: SemanticCodec decode (crates/core/src/models/codec.rs:202-239)
    of one cfg2 generate's 1,500 codes into [3000, 1024] features, seeded synthetic codec
    weights of the checkpoint's geometry; device time by CUDA events."""
    import itts_gpt as ig
    from itts_gpt.synth import make_codec_weights
    c = ig.SemanticCodec.from_weights(make_codec_weights(seed=77))
    ms = []
    for i in range(4):
        out = c.decode(codes)
        if i:
            ms.append(c.last_device_ms)
    c.close()
    dev = statistics.median(ms)
    return {"workload": f"SemanticCodec decode of {len(codes)} codes -> [{out.shape[0]}, {out.shape[1]}] fp32",
            "device_ms": dev, "codes_per_s": len(codes) / (dev * 1e-3)}


def bench_cfg1(cfg, gpt, w) -> dict:
    """batch 1, 32 conditioning latents + 64 text tokens (99 positions), 256
    greedy steps (repetition penalty 10); device time of prefill + decode."""
    import itts_gpt as ig
    from itts_gpt.synth import make_conds, make_text
    text = make_text(64, cfg.text_vocab, seed=11)
    conds = make_conds(cfg.d, N_CONDS, seed=12)
    kv = ig.KvCache(gpt, max_seq=N_CONDS + 64 + 3 + 256 + 8)
    p = ig.SamplingParams(greedy=True, max_mel_tokens=256)
    runs = []
    for i in range(4):
        codes = ig.generate_codes_after(gpt, ig.CodePrompt(text, conds, LANG, min_codes=256), kv, p,
                                        ig.SamplerRng(i))
        assert len(codes) == 256
        runs.append(gpt.last_timing())
    kv.close()
    pf, dc, nl = [statistics.median(x) for x in zip(*runs[1:])]
    return {"workload": "cfg1: batch 1, 32 conds + 64 text tokens, 256 greedy mel tokens (rep 10)",
            "ms_per_mel_token": (pf + dc) / 256, "decode_ms_per_step": dc / 255, "prefill_ms": pf,
            "mel_tokens_per_s": 256 / ((pf + dc) * 1e-3)}


def bench_cfg3(cfg, gpt, peaks, n_req=64, n_mel=600) -> dict:
    """64 requests (32 conds + text uniform in [16, 600]) in one batched
    generate of 600 sampled steps each (STOP masked, so every request runs all of them).
    Roofline: per decode step the int8 weights once plus the fp16 K/V of every live
    request, over the mean step time."""
    import itts_gpt as ig
    from itts_gpt.synth import make_conds, make_text
    lens = np.random.default_rng(3).integers(16, 601, n_req)
    prompts = [ig.CodePrompt(make_text(int(n), cfg.text_vocab, seed=900 + r),
                             make_conds(cfg.d, N_CONDS, seed=950 + r), LANG, min_codes=n_mel)
               for r, n in enumerate(lens)]
    params = ig.SamplingParams(max_mel_tokens=n_mel, **SAMPLING)
    kv = ig.KvCache(gpt, max_seq=int(lens.max()) + N_CONDS + 3 + n_mel + 8, max_batch=n_req)
    runs = []
    for i in range(3):
        out = ig.generate_batch(gpt, prompts, kv, params, [ig.SamplerRng(i * 100 + r) for r in range(n_req)])
        assert all(len(c) == n_mel for c in out)
        runs.append(gpt.last_timing())
    kv.close()
    pf, dc, nl = [statistics.median(x) for x in zip(*runs[1:])]
    T0 = lens + N_CONDS + 3
    steps = n_mel - 1
    kv_bytes = sum(kv_bytes_per_step(cfg, int(t) + s + 1) for t in T0 for s in range(0, steps, 50)) * 50 / steps
    step_bytes = cfg.weight_bytes() + kv_bytes
    ms_step = dc / steps
    achieved = step_bytes / (ms_step * 1e-3) / 1e9
    peak = float(peaks.get("hbm_gbs", 6650.0))
    return {"workload": f"cfg3: {n_req} requests, text U[16,600], {n_mel} sampled steps each (T 0.8, top-k 30, "
                        "top-p 0.8, rep 10), one batched generate",
            "mel_tokens_per_s": n_req * n_mel / ((pf + dc) * 1e-3), "prefill_ms": pf,
            "decode_ms_per_step": ms_step,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "algorithmic_bytes_per_step": step_bytes,
                         "bytes_formula": "514,144,936 int8 weight B + 122,880 B x KV positions of the 64 "
                                          "live requests (mean over the steps)"}}


def cfg5_requests(cfg, synth_path=None, n=1024, seed=5):
    """configs[4]'s queue: text lengths log-normal with median 80 (sigma 0.6, the spread the
    config leaves open), clipped to [8, 600]; mel length 3.5 x text clipped to 1800 (STOP
    masked until then, so every sentence yields exactly that many codes); cfg2's sampling."""
    import itts_gpt as ig
    from itts_gpt.serve import Request
    from itts_gpt.synth import make_conds, make_text
    rng = np.random.default_rng(seed)
    lens = np.clip(np.round(np.exp(np.log(80.0) + 0.6 * rng.standard_normal(n))), 8, 600).astype(int)
    reqs = []
    for i, L in enumerate(lens):
        mel = int(min(round(3.5 * L), 1800))
        prompt = ig.CodePrompt(make_text(int(L), cfg.text_vocab, seed=20000 + i),
                               make_conds(cfg.d, N_CONDS, seed=30000 + i, synth_path=synth_path), LANG,
                               min_codes=mel)
        reqs.append(Request(i, prompt, ig.SamplingParams(max_mel_tokens=mel, **SAMPLING), seed=40000 + i))
    return reqs


def bench_cfg5(cfg, w, rank, world, local_rank, max_batch=64, chunk=8) -> dict:
    """the 1,024-sentence queue served by one worker per GPU with continuous
    batching (itts_gpt.serve; up to 64 live requests per GPU), the queue shared by all ranks
    through the torch.distributed store.  Wall clock around the whole queue (synchronized
    on both sides; max over ranks), tokens summed over ranks."""
    import torch
    from itts_gpt.serve import Dispatcher, RequestQueue, StoreQueue, gpu_engine_factory
    reqs = cfg5_requests(cfg)
    max_seq = N_CONDS + 600 + 3 + 1800 + 8
    make = gpu_engine_factory(w, local_rank, max_batch=max_batch, max_seq=max_seq, chunk=chunk)
    # warm-up on this rank's own short queue: graphs, fp16 weight copies, allocations; the
    # worker keeps its engine (model replica and cache) for the timed queue
    d = Dispatcher([make], keep_engines=True)
    warm = d.run(RequestQueue(sorted(reqs, key=lambda r: r.prompt.min_codes)[:2 * max_batch]))
    assert all(r.error is None for r in warm.values()), d.workers[0].error
    if world > 1:
        import torch.distributed as dist
        store = dist.distributed_c10d._get_default_store()
        dist.barrier()
        queue = StoreQueue(store, "bench/cfg5/next", reqs)
    else:
        queue = RequestQueue(reqs)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    res = d.run(queue)
    torch.cuda.synchronize()
    secs = time.perf_counter() - t0
    d.close()
    sums = [sum(len(r.codes) for r in res.values()), len(res), sum(1 for r in res.values() if r.error)]
    secs_max = float(max_over_ranks([secs], world)[0])
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor(sums, dtype=torch.float64)
        dist.all_reduce(t)
        sums = [int(x) for x in t.tolist()]
    return {"workload": "cfg5: 1,024 sentences, text log-normal (median 80, sigma 0.6, [8, 600]), mel = "
                        "min(3.5 x text, 1800), cfg2 sampling; continuous batching, <= 64 live requests per "
                        "GPU, one shared queue",
            "mel_tokens_per_s": sums[0] / secs_max, "unit": "mel tokens/s (aggregate over GPUs)",
            "seconds": secs_max, "mel_tokens": sums[0], "sentences": sums[1], "errors": sums[2],
            "n_gpus": world, "timing": "wall clock around the queue, synchronized, max over ranks",
            "scaling": "strong (fixed 1,024-sentence queue)"}


def prefill_flops(cfg, lens) -> float:
    """FLOPs of a prefill of requests with `lens` positions: the 24 layers' linears on
    every position, the head on each request's last position, causal attention
    (QK^T and PV over keys 0..t of each query t)."""
    per_pos = 2.0 * cfg.n_layers * (3 * cfg.d * cfg.d + cfg.d * cfg.d + 2 * cfg.d * cfg.ff)
    head = 2.0 * cfg.d * cfg.mel_vocab
    attn = sum(2.0 * 2 * cfg.d * cfg.n_layers * T * (T + 1) / 2 for T in lens)
    return per_pos * sum(lens) + head * len(lens) + attn


def bench_prefill_cfg4(cfg, gpt, peaks, n_req=32, reps=3) -> dict:
    """configs[3]'s prefill: 32 prompts of 32 conditioning latents + 600 text tokens in
    one packed prefill (device time of the forward, CUDA events)."""
    import itts_gpt as ig
    prompts = []
    for r in range(n_req):
        text, conds = make_prompt(cfg, r)
        prompts.append(ig.CodePrompt(text, conds, LANG))
    T = N_CONDS + N_TEXT + 3
    kv = ig.KvCache(gpt, max_seq=T + 40, max_batch=n_req)
    ms = []
    for i in range(2 + reps):
        ig.prefill_batch(gpt, prompts, kv)
        if i >= 2:
            ms.append(gpt.last_timing()[0])
    # then configs[3]'s 32 decode steps of the 32 requests (a batched generate of 33 codes:
    # the first from the prefill, 32 from decode steps)
    params = ig.SamplingParams(max_mel_tokens=33, **SAMPLING)
    dec = []
    for i in range(3):
        out = ig.generate_batch(gpt, [ig.CodePrompt(p.text_tokens, p.conds, LANG, min_codes=33) for p in prompts],
                                kv, params, [ig.SamplerRng(i * 100 + r) for r in range(n_req)])
        assert all(len(c) == 33 for c in out)
        dec.append(gpt.last_timing()[1])
    kv.close()
    dev_ms = statistics.median(ms)
    dec_ms = statistics.median(dec[1:])
    flops = prefill_flops(cfg, [T] * n_req)
    peak = float(peaks.get("bf16_tflops_sustained", 1404.5))
    tf = flops / (dev_ms * 1e-3) / 1e12
    return {"workload": f"cfg4 prefill: {n_req} prompts x {T} positions in one packed prefill",
            "device_ms": dev_ms, "positions_per_s": n_req * T / (dev_ms * 1e-3),
            "tflops": tf, "flops": flops, "peak_tflops": peak,
            "peak_source": "measured sustained bf16" if "bf16_tflops_sustained" in peaks else "fallback",
            "frac": tf / peak,
            "decode_32_steps_ms": dec_ms, "decode_ms_per_step": dec_ms / 32,
            "decode_note": "32 decode steps of the 32 requests after the prefill (batched generate, "
                           "device time first sample through the last step)"}


def _bench_decode_forward(gpt, kv, kv_len, iters, nb=1):
    import ctypes as C
    from itts_gpt import _lib
    ms, n = C.c_float(), C.c_int32()
    rc = _lib.load_lib().itts_bench_decode_forward(gpt._h, kv._h, nb, kv_len, iters, C.byref(ms),
                                                   C.byref(n))
    if rc != 0:
        raise RuntimeError(_lib.last_error())
    return ms.value, n.value


def run_profile_case(args):
    """A small case for profilers: the full-size decode-step forward alone, 3 warm-up
    launches then `--profile-iters` timed ones, at KV length `--profile-decode`."""
    import itts_gpt as ig
    cfg, w = make_model()
    gpt = ig.Gpt.from_weights(w)
    nb = args.profile_nb
    kv = ig.KvCache(gpt, max_seq=args.profile_decode + 8, max_batch=nb)
    ms, n = _bench_decode_forward(gpt, kv, args.profile_decode, iters=args.profile_iters, nb=nb)
    print(json.dumps({"profile_case": "decode-step forward", "kv_len": args.profile_decode, "columns": nb,
                      "ms_per_step": ms, "launches_per_step": n}), flush=True)


def run_profile_prefill(args):
    """A small case for profilers: cfg2 prefills (635 positions) of one request, repeated."""
    import itts_gpt as ig
    cfg, w = make_model()
    gpt = ig.Gpt.from_weights(w)
    text, conds = make_prompt(cfg, 0)
    kv = ig.KvCache(gpt, max_seq=N_CONDS + N_TEXT + 3 + 8, max_batch=1)
    import time
    for i in range(args.profile_prefill):
        t0 = time.perf_counter()
        gpt.prefill(text, conds, LANG, kv)
        dt = time.perf_counter() - t0
    print(json.dumps({"profile_case": "cfg2 prefill", "positions": N_CONDS + N_TEXT + 3,
                      "repeats": args.profile_prefill, "last_wall_ms": 1000.0 * dt}), flush=True)


def run_profile_generate(args):
    """A case for profilers: cfg2's prompt and sampling, `--profile-generate` tokens (the
    decode step and the sampler launch once per token)."""
    import itts_gpt as ig
    cfg, w = make_model()
    gpt = ig.Gpt.from_weights(w)
    text, conds = make_prompt(cfg, 0)
    n = args.profile_generate
    kv = ig.KvCache(gpt, max_seq=N_CONDS + N_TEXT + 3 + n + 8, max_batch=1)
    params = ig.SamplingParams(max_mel_tokens=n, **SAMPLING)
    codes = ig.generate_codes_after(gpt, ig.CodePrompt(text, conds, LANG, min_codes=n), kv, params,
                                    ig.SamplerRng(1))
    pf, dc, nl = gpt.last_timing()
    print(json.dumps({"profile_case": "cfg2 generate", "tokens": len(codes), "prefill_ms": pf,
                      "decode_ms": dc, "ms_per_step": dc / max(1, len(codes) - 1)}), flush=True)


def run_profile_prefill_batch(args):
    """A case for profilers: the cfg4 prefill, N_REQ prompts of 32 conditioning latents +
    600 text tokens (635 positions each) in one packed prefill, run twice."""
    import itts_gpt as ig
    import torch
    cfg, w = make_model()
    gpt = ig.Gpt.from_weights(w)
    n = args.profile_prefill_batch
    prompts = []
    for r in range(n):
        text, conds = make_prompt(cfg, r)
        prompts.append(ig.CodePrompt(text, conds, LANG))
    kv = ig.KvCache(gpt, max_seq=N_CONDS + N_TEXT + 3 + 8, max_batch=n)
    for i in range(2):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        ig.prefill_batch(gpt, prompts, kv)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
    print(json.dumps({"profile_case": "cfg4 packed prefill", "requests": n,
                      "positions": n * (N_CONDS + N_TEXT + 3), "last_wall_ms": 1000.0 * dt}), flush=True)


# stage timeline events of xk_decode_kernel per layer (l >= 1) on cluster ranks other than 0
# the batch-1 kernel's stage stamps of one layer after the first (xk_decode.cu: trace())
XK_EVENTS = ["x pushed", "x gathered", "LayerNorm 1", "QKV tiles + push", "q/k/v in cluster",
             "attention records in cluster", "attention merged", "c_proj partials added", "h pushed",
             "h gathered", "LayerNorm 2", "c_fc tiles + push", "u in cluster", "mlp partials added"]


def run_profile_trace(args):
    """Stage timeline of one batch-1 decode step at KV length `--profile-trace`: per-CTA
    SM-cycle stamps (itts_bench_trace); each stage's duration is the gap to the previous
    stamp of the same CTA, median over all CTAs and layers 1 .. n_layers - 2."""
    import ctypes as C
    import numpy as np
    import itts_gpt as ig
    from itts_gpt import _lib
    cfg, w = make_model()
    gpt = ig.Gpt.from_weights(w)
    L = args.profile_trace
    kv = ig.KvCache(gpt, max_seq=L + 8, max_batch=1)
    if kv.decode_kernel(1) != "xk_decode_kernel":
        raise SystemExit("--profile-trace reads the event layout of xk_decode_kernel")
    lib = _lib.load_lib()
    n = 160 * 512
    out = np.zeros(n, np.uint64)
    g, e = C.c_int32(), C.c_int32()
    for _ in range(3):
        if lib.itts_bench_trace(gpt._h, kv._h, 1, L, out.ctypes.data, n, C.byref(g), C.byref(e)) != 0:
            raise RuntimeError(_lib.last_error())
    t = out[: g.value * e.value].reshape(g.value, e.value).astype(np.int64)
    nr = int((t[:, 0] > 0).sum())
    # stamp 0: CTA start; layer 0 (no x exchange) 1 .. E - 1; layers 1 .. nl - 1 from E on; then
    # x pushed / gathered, ln_f, final_norm, head; the last slot: CTA end
    E, first = len(XK_EVENTS), len(XK_EVENTS)
    nl = cfg.n_layers
    tail = first + (nl - 1) * E
    assert tail + 5 < e.value - 1
    lay = t[:nr, first - 1:tail]  # from layer 0's last stamp on
    d = np.diff(lay, axis=1).reshape(nr, nl - 1, E)[:, :-1, :]  # layers 1 .. nl - 2
    med = np.median(d.reshape(-1, E), axis=0)
    head = np.diff(t[:nr, tail - 1:tail + 5], axis=1)
    sm_mhz = 1965.0
    print(json.dumps({"profile_case": "decode-step stage timeline", "kv_len": L, "ctas": nr,
                      "cycles_per_layer": int(med.sum()), "us_per_layer_at_1965_mhz": round(float(med.sum()) / sm_mhz, 2),
                      "median_cycles_per_stage": {nm: int(med[i]) for i, nm in enumerate(XK_EVENTS)},
                      "median_cycles_start_to_embedding": int(np.median(t[:nr, 1] - t[:nr, 0])),
                      "median_cycles_layer_0": int(np.median(t[:nr, E - 1] - t[:nr, 1])),
                      "median_cycles_head": {nm: int(v) for nm, v in zip(
                          ["x pushed", "x gathered", "ln_f", "final_norm", "head tiles"], np.median(head, axis=0))},
                      "median_cycles_head_to_end": int(np.median(t[:nr, -1] - t[:nr, tail + 4])),
                      "median_cycles_start_to_end": int(np.median(t[:nr, -1] - t[:nr, 0]))}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="only the cfg2 headline (no cfg1/cfg3/cfg4/cfg5 keys)")
    ap.add_argument("--profile-decode", type=int, default=0, metavar="KV_LEN",
                    help="profiler case: only the decode-step forward at this KV length")
    ap.add_argument("--profile-iters", type=int, default=2)
    ap.add_argument("--profile-nb", type=int, default=1, help="batch columns of --profile-decode")
    ap.add_argument("--profile-prefill", type=int, default=0, metavar="REPEATS",
                    help="profiler case: only cfg2 prefills, this many")
    ap.add_argument("--profile-generate", type=int, default=0, metavar="TOKENS",
                    help="profiler case: one cfg2 generate of this many tokens")
    ap.add_argument("--profile-prefill-batch", type=int, default=0, metavar="N_REQ",
                    help="profiler case: the cfg4 packed prefill of N_REQ prompts, twice")
    ap.add_argument("--profile-trace", type=int, default=0, metavar="KV_LEN",
                    help="stage timeline of one batch-1 decode step at this KV length")
    args = ap.parse_args()
    if args.profile_trace > 0:
        run_profile_trace(args)
        return
    if args.profile_decode > 0:
        run_profile_case(args)
        return
    if args.profile_prefill > 0:
        run_profile_prefill(args)
        return
    if args.profile_prefill_batch > 0:
        run_profile_prefill_batch(args)
        return
    if args.profile_generate > 0:
        run_profile_generate(args)
        return
    rank, world, local_rank = dist_env()
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        else:
            run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
