"""Benchmark of the Qwen3 decoder forward on B200 (BASELINE.json metric: Qwen3-0.6B-shape tok/s, prefill and decode
b=64, at 1/2/4/8 GPUs, % HBM roofline).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...        (N > 1: one process per GPU)

Headline (value): BASELINE config 5 -- Qwen3-0.6B architecture, random N(0, 0.02) bf16 weights, greedy decode of 64
sequences per GPU, each with a 4096-token paged KV cache (16-token pages) prefilled from uniform-random ids through
the engine's own prefill; one step = one decode step of the 64 sequences (64 tokens per GPU). Sequences are
independent, so N GPUs run N x 64 (weak scaling, no collective on the hot path). The timed region replays the
captured decode step K times with every input resident on the device; e2e repeats the same K steps through the
public host API (ids copied in from pinned memory and next ids copied out every step). The KV cache (32 GB) is far
larger than L2, so no flush is needed between steps.

Also reported: BASELINE config 4 prefill (16 x 2048-token prompts per job, split over the GPUs), the decode-attention
kernel's HBM roofline (timed with CUDA events recorded inside the replayed step), clocks sampled during the timed
region, and the CPU reference (the oracle port) timed on a bounded sample on this host.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Qwen3-0.6B-shape tok/s (prefill, decode b=64) at 1/2/4/8 B200; % HBM roofline"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=248)
    p.add_argument("--warmup", type=int, default=8)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--batch", type=int, default=64, help="sequences per GPU")
    p.add_argument("--context", type=int, default=4096, help="prefilled KV tokens per sequence")
    p.add_argument("--no-prefill-bench", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-seconds", type=float, default=15.0, help="bounded CPU-baseline sample, seconds")
    p.add_argument("--layers", type=int, default=28, help="decoder layers (profiling cases use fewer)")
    p.add_argument("--no-decode", action="store_true", help="only the config-4 prefill part")
    p.add_argument("--prefill-batch", type=int, default=16, help="config-4 prompts per job")
    p.add_argument("--prefill-len", type=int, default=2048, help="config-4 prompt length")
    p.add_argument("--pipeline", action="store_true",
                   help="pipeline stage split instead of data parallelism: under torchrun each rank holds 28/N layers "
                        "of every sequence (not the headline)")
    p.add_argument("--microbatches", type=int, default=2, help="--pipeline: sequence groups in flight")
    p.add_argument("--op-bench", action="store_true",
                   help="operator benchmarks only (config 2 attention, config 4 GEMM shapes); one JSON line")
    p.add_argument("--attention-libraries", action="store_true",
                   help="--op-bench: also time the config-2 prefill through the attention libraries in the image "
                        "(flash_attn, flashinfer's Blackwell backends; the CUTLASS one compiles for about 2 minutes)")
    return p.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        if all(k in d for k in FALLBACK_PEAKS):
            return {k: float(d[k]) for k in FALLBACK_PEAKS}, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


class Dist:
    """One process per GPU (torchrun's RANK / LOCAL_RANK / WORLD_SIZE). Sequences are independent, so the process
    group carries only the timing barrier and the max-over-ranks reduction; `backend` is nccl on GPUs (gloo in the
    CPU tests of this plumbing). A rank that stops answering ends the others' next collective after `timeout_s`."""

    def __init__(self, backend: str = "nccl", timeout_s: float = 600.0):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.backend = backend
        self.timeout_s = timeout_s
        self.pg = None

    def init(self):
        import datetime

        import torch

        if self.backend == "nccl":
            torch.cuda.set_device(self.local)
        if self.world > 1:
            import torch.distributed as dist

            kw = {"device_id": torch.device(f"cuda:{self.local}")} if self.backend == "nccl" else {}
            dist.init_process_group(self.backend, timeout=datetime.timedelta(seconds=self.timeout_s), **kw)
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch

        dev = f"cuda:{self.local}" if self.backend == "nccl" else "cpu"
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


class ClockSampler:
    """nvidia-smi clocks and throttle reasons every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_ids):
        self.gpu_ids = gpu_ids
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200", "-i",
                 ",".join(self.gpu_ids)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        rows = [[x.strip() for x in ln.split(",")] for ln in out.splitlines() if ln.strip()]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if len(r) > 5 + i and r[5 + i] == "Active"})
        load = [s for s in sm if s > 0.5 * (max(sm) if sm else 0)]
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ---- the CPU reference (the oracle port; the reference's F# CPU path cannot be built here) ----------------------


def cpu_decode_sample(weights, cfg, context, seconds, max_steps=None):
    """Times CPU-reference decode steps of one sequence at `context` cached tokens (fp32 cache filled with random
    values: the cost of a step does not depend on them). Returns (tok/s, steps, seconds, threads)."""
    from oracle import oracle as O
    from rosylnalive_b200.rope import QWEN3_INV_FREQ_BITS  # a constant: nothing of liblrmcuda is loaded here

    steps_cap = max_steps or 10 ** 6
    max_pos = context + min(steps_cap, 4096) + 1
    cos, sin = O.rope_table(QWEN3_INV_FREQ_BITS, max_pos)  # the oracle's own T_spec builder
    oc = O.Config(cfg.layers, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.intermediate, cfg.vocab, cfg.eps,
                  max_pos)
    m = O.Model.from_hf(oc, weights, cos, sin)
    cache = O.Cache.new(oc, "f32", max_pos)
    g = np.random.default_rng(7)
    for arr in cache.keys + cache.values:
        arr[:context] = g.standard_normal((context, arr.shape[1]), dtype=np.float32)
    tok = 1
    t0 = time.perf_counter()
    n = 0
    while n < steps_cap and n + context < max_pos - 1:
        logits = O.forward(m, cache, context + n, [tok], "f32", logits_rows="last")
        tok = int(O.argmax_rows(logits, "f32")[0])
        n += 1
        if max_steps is None and time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return n / dt, n, dt, O.THREADS


def decode_config(B, ctx, world, layers):
    """The config-5 workload both arms report: our arm runs it whole, the reference arm times a bounded sample of it
    (described in its cpu_baseline.sample)."""
    return {"workload": f"config5: Qwen3-0.6B bf16 greedy decode, {B} seqs/GPU, {ctx}-token paged KV "
                        "(16-token pages), random-init weights N(0,0.02), random prompt ids"
                        + ("" if layers == 28 else f" [profiling case: {layers} layers]"),
            "model": "Qwen3-0.6B architecture", "global_batch": B * world, "seq_len": ctx,
            "parallelism": f"dp{world} (independent sequences per GPU, no collective)",
            "l2": "inputs larger than L2 (32 GB KV cache), no flush"}


def run_reference(args, dist):
    from rosylnalive_b200 import synthetic as S

    if dist.rank != 0:
        return
    cfg = S.QWEN3_0_6B
    weights = S.random_weights(cfg, seed=0)
    cpu_decode_sample(weights, cfg, args.context, 0, max_steps=max(1, args.warmup))
    tps, n, dt, threads = cpu_decode_sample(weights, cfg, args.context, 0, max_steps=max(1, args.steps))
    sample = (f"{n} CPU-reference decode steps of 1 sequence at {args.context} cached tokens (fp32 cache), "
              f"Qwen3-0.6B shape, {threads} threads; the config-5 step is 64 such sequences")
    line = {"impl": "reference", "metric": METRIC, "value": tps, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": n, "warmup": args.warmup, "ms_per_step": 1000 * dt / n, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": decode_config(args.batch, args.context, args.gpus, cfg.layers),
            "cpu_baseline": {"value": tps, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": tps, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---- our arm -------------------------------------------------------------------------------------------------


def run_ours(args, dist):
    import torch

    from rosylnalive_b200 import qwen as Qw
    from rosylnalive_b200 import rope as R
    from rosylnalive_b200 import synthetic as S

    pk, pk_kind = peaks()
    cfg = S.QWEN3_0_6B
    if args.layers != cfg.layers:
        import dataclasses

        cfg = dataclasses.replace(cfg, layers=args.layers)
    B, ctx, K, W = args.batch, args.context, args.steps, args.warmup
    weights = S.random_weights(cfg, seed=0)
    max_pos = (max(ctx + W + K + 16, args.prefill_len) + 15) // 16 * 16
    cos, sin = R.t_spec(R.QWEN3_INV_FREQ_BITS, max_pos)
    chunk = max(1, min(B, 32768 // ctx))
    pf_seqs = max(1, args.prefill_batch // dist.world)
    max_tokens = max(32768 if not args.no_decode else 0, pf_seqs * args.prefill_len)
    eng = Qw.QwenEngine(cfg, weights, cos, sin, device=dist.local, max_seqs=max(B, pf_seqs), max_tokens=max_tokens,
                        max_batch=B, max_pos=max_pos)
    stream = torch.cuda.ExternalStream(eng.stream)
    slots = np.arange(B, dtype=np.int32)

    def timed(fn):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dist.barrier()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            e0.record()
            fn()
            e1.record()
        e1.synchronize()
        torch.cuda.synchronize()
        dist.barrier()
        return dist.max(e0.elapsed_time(e1))

    if args.no_decode:
        prefill = prefill_bench(eng, cfg, dist, pk, stream, timed, args.prefill_batch, args.prefill_len)
        eng.close()
        if dist.rank == 0:
            print(json.dumps({"metric": METRIC, "value": prefill["value"], "unit": "tok/s", "n_gpus": dist.world,
                              "steps": prefill["timed_prefills"], "warmup": 2,
                              "ms_per_step": prefill["ms_per_prefill"],
                              "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                              "data": "synthetic", "config": {"workload": prefill["workload"],
                                                              "layers": cfg.layers},
                              "prefill": prefill}), flush=True)
        return

    # KV prefill from random ids (setup, not timed).
    prompts = S.random_prompts(cfg.vocab, B, ctx, seed=1000 + dist.rank)
    first = []
    for i in range(0, B, chunk):
        nxt, _ = eng.prefill(slots[i:i + chunk], list(prompts[i:i + chunk]))
        first.extend(nxt.tolist())
    eng.capture(slots, np.array(first, np.uint32))
    launches_per_step = eng.graph_kernels()
    eng.replay(W)
    eng.sync()
    start_len = ctx + W
    ids_at_start = eng.last_ids()

    gpu_ids = [torch.cuda.get_device_properties(i).uuid for i in range(torch.cuda.device_count())]
    sampler = ClockSampler([f"GPU-{u}" if not str(u).startswith("GPU-") else str(u) for u in gpu_ids]
                           if dist.rank == 0 else [])
    if dist.rank == 0:
        sampler.start()
        time.sleep(0.3)
    ms = timed(lambda: eng.replay(K))
    clocks = sampler.stop() if dist.rank == 0 else None
    value = B * dist.world * K / (ms / 1000.0)

    # e2e: the same K steps (rewound to the same positions) through the public host API.
    for s in slots:
        eng.truncate(int(s), start_len)
    cur = ids_at_start.copy()

    def e2e_steps():
        nonlocal cur
        for _ in range(K):
            cur, _ = eng.decode(slots, cur)

    ms_e2e = timed(e2e_steps)
    e2e_value = B * dist.world * K / (ms_e2e / 1000.0)
    # Bytes the e2e steps copy: in, the B ids each step (the slot list is already on the device, and the pages of
    # these positions were reserved by the replay above: truncate keeps them, so no page-table row is uploaded);
    # out, the B next ids and the 4-byte error word.
    e2e_h2d = 4 * B

    # Roofline of the dominant kernel (decode attention): events around each layer's launch inside the step.
    for s in slots:
        eng.truncate(int(s), start_len)
    eng.capture(slots, ids_at_start, time_attention=True)
    R_steps = min(K, 32)
    att_ms, att_bytes = [], []
    kvh, hd = cfg.kv_heads, cfg.head_dim
    for i in range(R_steps):
        eng.replay(1)
        per_layer = eng.attention_ms()
        keys = start_len + i + 1
        att_ms.extend(per_layer.tolist())
        # algorithmic bytes of one launch: K and V of every cached key (bf16) + q in + out (bf16)
        att_bytes.extend([B * keys * kvh * hd * 2 * 2 + 2 * B * cfg.heads * hd * 2] * len(per_layer))
    att_avg_ms = float(np.mean(att_ms))
    att_bytes_avg = float(np.mean(att_bytes))
    achieved = att_bytes_avg / (att_avg_ms / 1000.0) / 1e9
    traffic = profile_traffic("decode_attention", att_bytes_avg)
    roofline = {"kernel": "decode_attn_kernel + decode_combine_kernel", "bound": "hbm", "achieved": achieved,
                "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"], "traffic": traffic,
                "peak_source": f"{pk_kind} hbm_gbs", "algorithmic_bytes_per_launch": att_bytes_avg,
                "avg_launch_ms": att_avg_ms, "launches_timed": len(att_ms),
                "share_of_step": float(np.sum(att_ms) / R_steps) / (ms / K)}
    # Whole-step HBM roofline: algorithmic bytes of one decode step (weights once, KV of every key, logits).
    step_bytes = (weights_bytes(cfg) + B * (start_len + K / 2) * cfg.layers * kvh * hd * 2 * 2
                  + B * cfg.vocab * 4)
    step_roof = {"algorithmic_bytes_per_step": step_bytes,
                 "achieved_gbs": step_bytes / (ms / K / 1000.0) / 1e9,
                 "frac": step_bytes / (ms / K / 1000.0) / 1e9 / pk["hbm_gbs"]}

    prefill = None
    if not args.no_prefill_bench:
        prefill = prefill_bench(eng, cfg, dist, pk, stream, timed, args.prefill_batch, args.prefill_len)
    eng.close()

    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        tps, n, dt, threads = cpu_decode_sample(weights, cfg, ctx, args.cpu_seconds)
        cpu = {"value": tps, "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"{n} CPU-reference (oracle port) decode steps of 1 sequence at {ctx} cached tokens, "
                         f"{dt:.1f} s on {threads} threads"}

    if dist.rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": dist.world, "steps": K, "warmup": W,
                "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic",
                "config": decode_config(B, ctx, dist.world, cfg.layers),
                "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": e2e_h2d,
                        "d2h_bytes_per_step": 4 * B + 4},
                "gpu_launches": launches_per_step * K * dist.world, "roofline": roofline, "step_roofline": step_roof,
                "prefill": prefill, "cpu_baseline": cpu, "clocks": clocks}
        print(json.dumps(line), flush=True)


def run_pipeline(args, dist):
    """The pipeline stage split (the reference's planned StagePipeline; not the headline): rank r holds
    stage r of the 28 layers (rosylnalive_b200.pipeline.split_layers) for all B x N sequences; the fp32 residual
    crosses ranks with NCCL send/recv, the next ids return to rank 0, and the sequences run in `microbatches` groups
    so the stages work concurrently. Setup prefills the KV caches through the same pipeline; the timed region is
    K decode steps of every group, timed on rank 0's device with a barrier and max over ranks."""
    import torch

    from rosylnalive_b200 import pipeline as PL
    from rosylnalive_b200 import qwen as Qw
    from rosylnalive_b200 import rope as R
    from rosylnalive_b200 import synthetic as S

    cfg = S.QWEN3_0_6B
    N, B, ctx, K, W = dist.world, args.batch * dist.world, args.context, args.steps, args.warmup
    first, end = PL.split_layers(cfg.layers, N)[dist.rank]
    max_pos = (ctx + W + K + 16 + 15) // 16 * 16
    cos, sin = R.t_spec(R.QWEN3_INV_FREQ_BITS, max_pos)
    weights = {k: v for k, v in S.random_weights(cfg, seed=0).items()}
    groups = max(1, args.microbatches)
    per_group = (B + groups - 1) // groups
    eng = Qw.QwenEngine(cfg, weights, cos, sin, device=dist.local, max_seqs=B, max_tokens=32768,
                        max_batch=per_group, max_pos=max_pos, stage=(first, end))
    dev = f"cuda:{dist.local}"
    pipe = PL.DistPipeline(eng, dist.rank, N, dev)
    prompts = list(S.random_prompts(cfg.vocab, B, ctx, seed=1000))
    # setup: prefill (in groups of at most 32,768 tokens) and W warm-up steps through the pipeline
    t0 = time.time()
    pipe.prefill(prompts, microbatches=max(groups, (B * ctx + 32767) // 32768))
    pipe.decode_steps(W, microbatches=groups)
    setup_s = time.time() - t0
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    ids = pipe.decode_steps(K, microbatches=groups)
    e1.record()
    e1.synchronize()
    dist.barrier()
    ms = dist.max(e0.elapsed_time(e1))
    eng.close()
    if dist.rank == 0:
        print(json.dumps({"metric": METRIC, "value": B * K / (ms / 1000.0), "unit": "tok/s", "n_gpus": N,
                          "steps": K, "warmup": W, "ms_per_step": ms / K, "higher_is_better": True,
                          "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                          "config": {"workload": f"config5 decode through a {N}-stage pipeline: {B} sequences, "
                                                 f"{ctx}-token paged KV, {groups} microbatches",
                                     "parallelism": f"pp{N} (layers {PL.split_layers(cfg.layers, N)})"},
                          "mode": "pipeline", "setup_s": setup_s,
                          "ids_checksum": int(np.sum(ids)) if ids is not None else None}), flush=True)


def weights_bytes(cfg) -> int:
    from rosylnalive_b200.executor import weight_shapes

    return int(sum(np.prod(s) for s in weight_shapes(cfg).values()) * 2)


def profile_traffic(kernel: str, algorithmic_bytes: float):
    """DRAM bytes per launch from the committed ncu summary of the kernel (profiles/<kernel>_traffic.json: bytes
    per algorithmic byte, measured on a smaller case), scaled to this launch; None when no summary exists."""
    path = os.path.join(ROOT, "profiles", f"{kernel}_traffic.json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        d = json.load(f)
    return float(d["dram_bytes_per_algorithmic_byte"]) * algorithmic_bytes


def prefill_bench(eng, cfg, dist, pk, stream, timed, batch=16, L=2048):
    """16 x 2048-token prompts per job, 16 / N per GPU (strong scaling)."""
    from rosylnalive_b200 import synthetic as S

    nseq = max(1, batch // dist.world)
    prompts = list(S.random_prompts(cfg.vocab, nseq, L, seed=2000 + dist.rank))
    slots = np.arange(nseq, dtype=np.int32)
    for _ in range(2):
        eng.prefill(slots, prompts)
    # the median of individually timed prefills (max over ranks each), steadier than one short window; clocks are
    # sampled meanwhile on rank 0
    import torch

    sampler = None
    if dist.rank == 0:
        u = str(torch.cuda.get_device_properties(torch.cuda.current_device()).uuid)
        sampler = ClockSampler([u if u.startswith("GPU-") else f"GPU-{u}"])
        sampler.start()
    samples = [timed(lambda: eng.prefill(slots, prompts)) for _ in range(8)]
    clocks = sampler.stop() if sampler else None
    ms = statistics.median(samples)
    tokens_job = nseq * dist.world * L
    # algorithmic FLOPs per GPU (the reference's OpCost conventions): GEMMs 2 * params * tokens, attention
    # 4 * hd * (causal pairs) per head and layer, lm_head on the last rows
    from rosylnalive_b200.executor import weight_shapes

    layer_params = sum(np.prod(s) for n, s in weight_shapes(cfg).items() if ".layers." in n and s.__len__() == 2)
    gemm_flops = 2 * layer_params * nseq * L
    attn_flops = cfg.layers * cfg.heads * nseq * (L * (L + 1) / 2) * (4 * cfg.head_dim)
    head_flops = 2 * cfg.vocab * cfg.hidden * nseq
    flops = gemm_flops + attn_flops + head_flops
    achieved = flops / (ms / 1000.0) / 1e12
    return {"value": tokens_job / (ms / 1000.0), "unit": "tok/s", "ms_per_prefill": ms,
            "ms_min_max": [min(samples), max(samples)], "timed_prefills": len(samples), "clocks": clocks,
            "workload": f"config4: {nseq * dist.world} x {L}-token prompts, {nseq} per GPU (strong scaling)",
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": pk["bf16_tflops_sustained"],
                         "unit": "TFLOP/s", "frac": achieved / pk["bf16_tflops_sustained"],
                         "peak_source": "measured bf16_tflops_sustained: a prefill is tens of ms of back-to-back "
                                        "tensor work under the power cap",
                         "frac_of_burst": achieved / pk["bf16_tflops"], "burst_peak": pk["bf16_tflops"],
                         "flops_per_gpu": flops,
                         "note": "whole prefill (GEMMs + attention) against the measured bf16 GEMM peak"}}


def op_bench(libraries=False):
    """Operator benchmarks on cuda:0 through the C ABI (one JSON line; not the headline): BASELINE config 2 (the
    standalone GQA attention op: batch 8, 16 query / 8 KV heads, head_dim 128, causal prefill of 2048 tokens and
    decode of one token over 4096 cached ones, bf16 Q/K/V ~ N(0, 1)) and the four prefill GEMM shapes of config 4
    (M = 32768 tokens) on one CTA per tile, on CTA pairs, and through torch.matmul (cuBLAS) for comparison. Each
    timing is the median of 20 launches with a 256 MB buffer written between launches (L2 flush)."""
    import torch

    from rosylnalive_b200 import ops

    ops.set_device(0)
    torch.cuda.set_device(0)
    pk, src = peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(0)

    def med_ms(fn, reps=20):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(reps):
            flush.zero_()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            ts.append(s.elapsed_time(e))
        return statistics.median(ts)

    res = {"metric": "operator benchmarks (BASELINE config 2 attention, config 4 GEMM shapes)", "impl": "ours",
           "peaks": {**pk, "source": src}}
    # config 2, prefill: packed sequences of 2048 tokens
    B, L, QH, KVH = 8, 2048, 16, 8
    T = B * L
    q = torch.randn(T, QH, 128, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(T, KVH, 128, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(T, KVH, 128, device="cuda", generator=g).to(torch.bfloat16)
    out = torch.empty(T, QH, 128, device="cuda", dtype=torch.bfloat16)
    cu = torch.arange(0, T + 1, L, device="cuda", dtype=torch.int32)
    ms = med_ms(lambda: ops.prefill_attention(q, k, v, out, cu, L, 1.0 / 128 ** 0.5))
    flops = 4.0 * 128 * QH * B * L * (L + 1) / 2
    res["attention_prefill"] = {"shape": "8 x 2048, 16/8 heads, causal", "ms": ms,
                                "tflops": flops / ms / 1e9, "frac_of_bf16_peak": flops / ms / 1e9 / pk["bf16_tflops"],
                                "flops": flops, "note": "causal FLOPs 4*d*heads*sum(L(L+1)/2)"}
    if libraries:
        res["attention_prefill_libraries"] = library_attention(q, k, v, cu, L, QH, KVH, flops, med_ms)
        del q, k, v, out
        res["attention_decode_config5_libraries"] = library_decode(QH, KVH, med_ms, pk, g)
    # config 2, decode: one query per sequence over 4096 cached tokens in 16-token pages
    C = 4096
    pages = C // 16
    pool = torch.randn(B * pages, KVH, 2, 16, 128, device="cuda", generator=g).to(torch.bfloat16)
    table = torch.randperm(B * pages, device="cuda", generator=g).to(torch.int32).view(B, pages)
    lens = torch.full((B,), C, dtype=torch.int32, device="cuda")
    slots = torch.arange(B, dtype=torch.int32, device="cuda")
    dq = torch.randn(B, QH, 128, device="cuda", generator=g).to(torch.bfloat16)
    dout = torch.empty(B, QH, 128, device="cuda", dtype=torch.bfloat16)
    want_ctas = 4 * 148
    pps = max(1, -(-pages // max(1, -(-want_ctas // (B * KVH)))))
    ws = torch.empty(ops.decode_attention_workspace(B, KVH, pages, pps) // 4, device="cuda")
    ms = med_ms(lambda: ops.decode_attention(dq, pool, table, lens, slots, dout, ws, pps, 1.0 / 128 ** 0.5))
    nbytes = B * C * KVH * 2 * 128 * 2 + dq.numel() * 2 + dout.numel() * 2
    res["attention_decode"] = {"shape": "8 x 1 query over 4096 cached tokens, 16/8 heads", "ms": ms,
                               "gbs": nbytes / ms / 1e6, "frac_of_hbm": nbytes / ms / 1e6 / pk["hbm_gbs"],
                               "bytes": nbytes, "pages_per_split": pps}
    # config 4 prefill GEMM shapes
    M = 32768
    shapes = [("q/k/v", 4096, 1024, ops.GEMM_BF16), ("o_proj + residual", 1024, 2048, ops.GEMM_RESID),
              ("gate/up + SwiGLU", 6144, 1024, ops.GEMM_SWIGLU), ("down + residual", 1024, 3072, ops.GEMM_RESID)]
    rows = []
    for name, n, kk, epi in shapes:
        a = torch.randn(M, kk, device="cuda", generator=g).to(torch.bfloat16)
        b = (torch.randn(n, kk, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
        if epi == ops.GEMM_SWIGLU:
            o = torch.empty(M, n // 2, device="cuda", dtype=torch.bfloat16)
        elif epi == ops.GEMM_BF16:
            o = torch.empty(M, n, device="cuda", dtype=torch.bfloat16)
        else:
            o = torch.zeros(M, n, device="cuda")
        r = o if epi == ops.GEMM_RESID else None
        fl = 2.0 * M * n * kk
        row = {"gemm": name, "m": M, "n": n, "k": kk}
        for label, pair in (("one_cta", 1), ("cta_pair", 2)):
            ms = med_ms(lambda: ops.gemm(a, b, o, epi, resid=r, bn=256, cta_pair=pair))
            row[label + "_tflops"] = fl / ms / 1e9
        ms = med_ms(lambda: torch.matmul(a, b.T))
        row["torch_matmul_bf16_out_tflops"] = fl / ms / 1e9
        row["cta_pair_frac_of_bf16_peak"] = row["cta_pair_tflops"] / pk["bf16_tflops"]
        rows.append(row)
    res["gemm_config4"] = rows
    print(json.dumps(res), flush=True)


def library_attention(q, k, v, cu, L, QH, KVH, flops, med_ms):
    """The same config-2 causal prefill through the attention libraries in the image, for comparison only (they are
    not part of this backend): flash_attn's varlen kernel and flashinfer's ragged prefill on its Blackwell backends.
    A backend that does not build or run here reports why."""
    import torch

    out = {}
    scale = 1.0 / 128 ** 0.5
    try:
        from flash_attn import flash_attn_varlen_func

        ms = med_ms(lambda: flash_attn_varlen_func(q, k, v, cu, cu, L, L, softmax_scale=scale, causal=True))
        out["flash_attn_varlen"] = {"ms": ms, "tflops": flops / ms / 1e9}
    except Exception as e:  # noqa: BLE001 - report any failure of an optional comparison
        out["flash_attn_varlen"] = {"unavailable": f"{type(e).__name__}: {str(e)[:160]}"}
    try:
        import flashinfer
    except Exception as e:  # noqa: BLE001
        out["flashinfer"] = {"unavailable": f"{type(e).__name__}: {str(e)[:160]}"}
        return out
    ws = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for backend in ("cutlass", "cute-dsl", "fa2"):
        try:
            w = flashinfer.BatchPrefillWithRaggedKVCacheWrapper(ws, "NHD", backend=backend)
            w.plan(cu, cu, QH, KVH, 128, causal=True, q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16,
                   sm_scale=scale)
            ms = med_ms(lambda: w.run(q, k, v))
            out[f"flashinfer_{backend}"] = {"ms": ms, "tflops": flops / ms / 1e9}
        except Exception as e:  # noqa: BLE001
            out[f"flashinfer_{backend}"] = {"unavailable": f"{type(e).__name__}: {str(e)[:160]}"}
    return out


def library_decode(QH, KVH, med_ms, pk, g):
    """Decode attention at the config-5 shape (64 sequences, 4096 cached tokens in 16-token pages, one query each):
    this backend's operator (32 pages a split, as the engine) beside flashinfer's paged decode on the same pages,
    copied into its [page][K/V][kv head][16][128] layout. For comparison only."""
    import torch

    from rosylnalive_b200 import ops

    B, C, P = 64, 4096, 16
    pages = C // P
    nbytes = B * C * KVH * 2 * 128 * 2 + 2 * B * QH * 128 * 2
    pool = torch.randn(B * pages, KVH, 2, P, 128, device="cuda", generator=g).to(torch.bfloat16)
    table = torch.randperm(B * pages, device="cuda", generator=g).to(torch.int32).view(B, pages)
    lens = torch.full((B,), C, dtype=torch.int32, device="cuda")
    slots = torch.arange(B, dtype=torch.int32, device="cuda")
    q = torch.randn(B, QH, 128, device="cuda", generator=g).to(torch.bfloat16)
    out = torch.empty(B, QH, 128, device="cuda", dtype=torch.bfloat16)
    ws = torch.empty(ops.decode_attention_workspace(B, KVH, pages, 32) // 4, device="cuda")
    res = {"shape": "64 x 1 query over 4096 cached tokens, 16/8 heads, 16-token pages", "bytes": nbytes}
    ms = med_ms(lambda: ops.decode_attention(q, pool, table, lens, slots, out, ws, 32, 1.0 / 128 ** 0.5))
    res["ours"] = {"ms": ms, "gbs": nbytes / ms / 1e6, "frac_of_hbm": nbytes / ms / 1e6 / pk["hbm_gbs"]}
    # one split a row: 512 CTAs, all resident, each writing its output (no combine launch)
    ws1 = torch.empty(ops.decode_attention_workspace(B, KVH, pages, pages) // 4, device="cuda")
    ms = med_ms(lambda: ops.decode_attention(q, pool, table, lens, slots, out, ws1, pages, 1.0 / 128 ** 0.5))
    res["ours_one_split"] = {"ms": ms, "gbs": nbytes / ms / 1e6, "frac_of_hbm": nbytes / ms / 1e6 / pk["hbm_gbs"]}
    try:
        import flashinfer
    except Exception as e:  # noqa: BLE001 - report any failure of an optional comparison
        res["flashinfer"] = {"unavailable": f"{type(e).__name__}: {str(e)[:160]}"}
        return res
    cache = pool.permute(0, 2, 1, 3, 4).contiguous()  # [page][K/V][kv head][16][128]
    indptr = torch.arange(0, B * pages + 1, pages, device="cuda", dtype=torch.int32)
    indices = table.reshape(-1).contiguous()
    last = torch.full((B,), P, dtype=torch.int32, device="cuda")
    fws = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for backend, tc in (("fa2", False), ("fa2", True), ("trtllm-gen", False)):
        key = f"flashinfer_{backend}" + ("_tensor_cores" if tc else "")
        try:
            w = flashinfer.BatchDecodeWithPagedKVCacheWrapper(fws, "HND", use_tensor_cores=tc, backend=backend)
            w.plan(indptr, indices, last, QH, KVH, 128, P, q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16,
                   sm_scale=1.0 / 128 ** 0.5)
            ms = med_ms(lambda: w.run(q, cache))
            res[key] = {"ms": ms, "gbs": nbytes / ms / 1e6}
        except Exception as e:  # noqa: BLE001
            res[key] = {"unavailable": f"{type(e).__name__}: {str(e)[:160]}"}
    return res


def main():
    args = parse()
    if args.op_bench:
        op_bench(libraries=args.attention_libraries)
        return
    dist = Dist()
    if args.impl == "reference":
        run_reference(args, dist)
        return
    dist.init()
    try:
        if args.pipeline:
            run_pipeline(args, dist)
        else:
            run_ours(args, dist)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
