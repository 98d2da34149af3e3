"""Benchmark: CDB decode throughput of the B200 engine -> one JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--requests R]

Workload: Ouro-1.4B architecture (24 layers, hidden 2048, 16x128
MHA heads, SwiGLU 5632, vocab 49152, 4 recurrent steps), random-init bf16; 256 concurrent
requests, prompt lengths LogNormal(median 200, sigma 0.8, cap 2048), output lengths
LogNormal(median 250, sigma 0.9, cap 1024), token ids uniform; per-token exit depths replayed
from a seeded categorical over {1,2,3,4} with p=(0.2,0.3,0.3,0.2); kv_policy single, block 16,
refill on. All inputs are seeded synthetic data (numpy default_rng), no dataset.

A step is one ``generate_batch`` over the whole request set (prefill included, as the
reference's ``generated_tokens / wall_time`` metric, ``benchmarks/metrics.py:274-278``).
``value`` is generated tokens / device time (CUDA events on the engine stream, max over ranks);
``e2e`` is the same through the public API measured on the host clock, which includes the prompt
upload and the token read-back of every step. Under torchrun the ranks are independent engine
replicas serving one seeded trace of 256 x N requests, request i on rank i mod N (``scaling:
weak``: 256 concurrent requests per GPU); nothing crosses GPUs inside the timed region.

``--config 4`` runs BASELINE config 4 instead: one 8192-request trace with seeded Poisson arrivals
at 200 requests/s in total (lengths and depths as config 1), request i on rank i mod N with its
arrival offset, one pass; whole-box tokens/s = all generated tokens / the slowest rank's time
(``scaling: strong``: the trace is fixed, more GPUs share it).

``--impl reference`` times the CPU restatement of the reference engine (``oracle/``, the only
place bench.py runs it) on the host cores over a bounded sample of the same workload (the first
4 config-1 requests at their full prompt lengths, 16 new tokens each); the b200 line reports its
own tokens/s on that same sample (``same_sample``) beside it.

``--engine cb`` times the full-depth continuous-batching baseline (``ContinuousBatchingEngine``,
the reference's CB comparison engine) on the same kernels, graphs and workload, and prints its
own line with ``"engine": "cb"``; every token then runs all 4 recurrent steps.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tokens/s/GPU, Ouro-1.4B CDB; paged-attn HBM GB/s vs 8 TB/s peak"
UNIT = "tokens/s"
OURO_1P4B = dict(
    vocab_size=49152, hidden_size=2048, intermediate_size=5632, num_hidden_layers=24, num_attention_heads=16,
    num_key_value_heads=16, head_dim=128, rope_theta=10000.0, rms_norm_eps=1e-6, max_position_embeddings=4096,
    total_ut_steps=4,
)
DEPTH_P = (0.2, 0.3, 0.3, 0.2)


def parse() -> argparse.Namespace:
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="b200", choices=["b200", "reference"])
    p.add_argument("--requests", type=int, default=256)
    p.add_argument("--out-cap", type=int, default=1024, help="cap on output lengths (smaller = profiling case)")
    p.add_argument("--no-graph", action="store_true")
    p.add_argument("--lm-head", default="fused", choices=["fused", "gemm"],
                   help="LM head + argmax as one tcgen05 GEMM (fused) or a GEMM then an argmax kernel")
    p.add_argument("--num-blocks", type=int, default=16384, help="KV pool blocks (small for profiler captures)")
    p.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU oracle timing (profiling runs)")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--engine", default="cdb", choices=["cdb", "cb"],
                   help="cdb: the CDB engine (the headline); cb: the full-depth continuous-batching baseline")
    p.add_argument("--config", type=int, default=1, choices=[1, 2, 3, 4],
                   help="BASELINE config: 1 (the headline) Ouro-1.4B, 256 concurrent requests per GPU; 2 Ouro-2.6B, "
                   "last_exited KV, Poisson 20 req/s; 3 Huginn-0125, S=32; 4 the 8192-request Poisson trace")
    p.add_argument("--no-refill", action="store_true", help="config 2: the no-refill (wave) arm")
    p.add_argument("--rate", type=float, default=200.0, help="config 4: total arrival rate, requests/s")
    p.add_argument("--trace-requests", type=int, default=8192, help="config 4: requests in the trace")
    return p.parse_args()


def dist_env() -> tuple[int, int, int]:
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def aggregate(dev_s: float, wall_s: float, tokens: float, device) -> tuple[float, float, float]:
    """Whole-job numbers across replicas: max over ranks of the times, sum of generated tokens.

    Runs after the timed region; with one process it returns its inputs.
    """

    import torch.distributed as dist

    if not dist.is_initialized() or dist.get_world_size() == 1:
        return dev_s, wall_s, tokens
    t = torch.tensor([dev_s, wall_s], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    n = torch.tensor([tokens], dtype=torch.float64, device=device)
    dist.all_reduce(n, op=dist.ReduceOp.SUM)
    return float(t[0]), float(t[1]), float(n[0])


def replica_seed(seed: int, rank: int) -> int:
    """Seed of the trace every rank draws from (one trace, split round-robin by ``shard``)."""

    del rank
    return seed


def workload(seed: int, n: int, out_cap: int):
    from oracle.workloads import ouro_lognormal_workload

    return ouro_lognormal_workload(n, vocab_size=OURO_1P4B["vocab_size"], seed=seed, out_cap=out_cap, depth_probs=DEPTH_P)


def shard(items: list, rank: int, world: int) -> list:
    """Request i of a trace goes to rank i mod world."""

    return items[rank::world]


def rank_workload(seed: int, per_rank: int, out_cap: int, rank: int, world: int):
    """This rank's share of one seeded trace of ``per_rank * world`` requests (the config-1 mix)."""

    prompts, max_new, depths = workload(replica_seed(seed, rank), per_rank * world, out_cap)
    return shard(prompts, rank, world), shard(max_new, rank, world), shard(depths, rank, world)


def config_workload(args, rank: int, world: int):
    """(prompts, max_new_tokens, exit_depths, arrival offsets or None) of this rank for ``--config``."""

    import numpy as np

    from oracle.workloads import huginn_workload, ouro_lognormal_workload, poisson_arrival_offsets

    if args.config == 3:
        p, m, d = huginn_workload(args.requests * world, vocab_size=65536, seed=args.seed, new_tokens=256, max_depth=32)
        return shard(p, rank, world), shard(m, rank, world), shard(d, rank, world), None
    if args.config == 2:
        n = args.requests * world
        p, m, d = ouro_lognormal_workload(n, vocab_size=OURO_1P4B["vocab_size"], seed=args.seed, out_cap=args.out_cap,
                                          depth_probs=DEPTH_P2)
        arr = poisson_arrival_offsets(np.random.default_rng(args.seed + 1), n, 20.0 * world)
        return shard(p, rank, world), shard(m, rank, world), shard(d, rank, world), shard(arr, rank, world)
    p, m, d = rank_workload(args.seed, args.requests, args.out_cap, rank, world)
    return p, m, d, None


def config4_trace(seed: int, n: int, rate: float, out_cap: int):
    """n requests with the config-1 lengths and depths and seeded Poisson arrival
    offsets at ``rate`` requests/s in total."""

    import numpy as np

    from oracle.workloads import poisson_arrival_offsets

    prompts, max_new, depths = workload(seed, n, out_cap)
    arrivals = poisson_arrival_offsets(np.random.default_rng(seed + 1), n, rate)
    return prompts, max_new, depths, arrivals


class ClockSampler:
    """nvidia-smi SM clocks / throttle reasons sampled every 200 ms while running."""

    def __init__(self, index: int) -> None:
        self.index = index
        self.proc = None

    def __enter__(self):
        q = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            out, _ = self.proc.communicate(timeout=10)
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9], strict=True):
                if flag.lower() == "active":
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": mx or None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


OURO_2P6B = {**OURO_1P4B, "num_hidden_layers": 48}
DEPTH_P2 = (0.1, 0.2, 0.3, 0.4)
# KV blocks of config 2 (48 layers x 4 last_exited slots: 25 MB per block) within ~140 GB of HBM
CONFIG2_BLOCKS = 5600


def build_engine(args, device):
    from continuous_depth_batching_b200 import (
        ContinuousDepthBatchingConfig,
        ContinuousDepthBatchingEngine,
        HuginnForCausalLM,
        OuroForCausalLM,
        OuroShape,
    )
    from continuous_depth_batching_b200.huginn import HuginnShape

    config = getattr(args, "config", 1)
    common = dict(block_size=16, synthetic_exit_replay=True, use_async_batching=False, use_cuda_graph=not args.no_graph,
                  max_model_len=4096, max_num_seqs=256)
    if config == 3:
        shape = HuginnShape()  # Huginn-0125: 2/4/2 blocks, 5280 wide, 55 x 96 heads, SwiGLU 17920, vocab 65536
        model = HuginnForCausalLM.random_init(shape, seed=1234, dtype=torch.bfloat16, device=device)
        cfg = ContinuousDepthBatchingConfig(num_blocks=args.num_blocks, max_recurrent_steps=32, refill=True,
                                            kv_policy="single", **common)
    elif config == 2:
        shape = OuroShape(**OURO_2P6B)
        model = OuroForCausalLM.random_init(shape, seed=1234, dtype=torch.bfloat16, device=device)
        cfg = ContinuousDepthBatchingConfig(num_blocks=min(args.num_blocks, CONFIG2_BLOCKS), max_recurrent_steps=4,
                                            refill=not args.no_refill, kv_policy="last_exited",
                                            kv_pressure_mode="reserve", **common)
    else:
        shape = OuroShape(**OURO_1P4B)
        model = OuroForCausalLM.random_init(shape, seed=1234, dtype=torch.bfloat16, device=device)
        cfg = ContinuousDepthBatchingConfig(num_blocks=args.num_blocks, max_recurrent_steps=4, refill=True,
                                            kv_policy="single", **common)
    eng = ContinuousDepthBatchingEngine.from_model(
        model, cfg, device=device, fused_lm_head=getattr(args, "lm_head", "fused") == "fused"
    )
    del model
    return eng, shape


# DRAM bytes per algorithmic byte of decode_attn_kernel<128,4> with the fused append, from one ncu
# capture of a launch of 128 rows x ~1055-token contexts (kernel_bench attention --rows 128
# --context 1024 --append 2): dram__bytes_read.sum 1.117724 GB + dram__bytes_write.sum 5.687 MB
# over 1,108,149,464 algorithmic bytes. Traffic grows with the pages a launch streams, so a bench
# launch's traffic is its algorithmic bytes times this ratio.
ATTN_TRAFFIC_PER_ALGO_BYTE = (1.117724e9 + 5.687296e6) / 1108149464


def attention_roofline(eng, shape, launches: list[tuple[list[int], list[int]]], peak_gbs: float) -> dict:
    """Time the paged decode-attention kernel alone over recorded launch shapes (CUDA events).

    Each recorded recurrent launch (rows' slots and positions) is replayed as the per-layer
    attention launch the engine makes: RoPE of q and k, the KV append at position p and attention
    over 0..p in one kernel (append=2), on the engine stream; achieved = algorithmic bytes (cache
    rows 0..p-1 read, the new k/v read and written, q read, o written) / mean launch time.
    """

    from continuous_depth_batching_b200.kernel_bench import attention_bytes

    r = eng.runner
    D, H = shape.head_dim, shape.num_attention_heads
    rope_mode = 2 if D == 96 else 1  # Huginn's interleaved fp32 RoPE tables, else Ouro's split-half
    total_bytes, total_ms, n = 0.0, 0.0, 0
    stream = r.stream
    for slots, pos in launches:
        b = len(pos)
        meta = r.upload([slots, pos])
        meta = meta.view(2, b)
        with torch.cuda.stream(stream):
            r._plan(meta[1], b, 1)
        algo = attention_bytes(pos, H, D, append=True)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 10
        with torch.cuda.stream(stream):
            r._attention(b, 0, meta[0], meta[1], 2, rope_mode)  # warm
            start.record(stream)
            for _ in range(reps):
                r._attention(b, 0, meta[0], meta[1], 2, rope_mode)
            end.record(stream)
        end.synchronize()
        ms = start.elapsed_time(end) / reps
        total_bytes += algo
        total_ms += ms
        n += 1
    per_launch_bytes = total_bytes / n
    per_launch_ms = total_ms / n
    achieved = per_launch_bytes / (per_launch_ms * 1e-3) / 1e9
    return {
        "bound": "hbm",
        "achieved": round(achieved, 1),
        "peak": peak_gbs,
        "unit": "GB/s",
        "frac": round(achieved / peak_gbs, 4),
        "traffic": int(per_launch_bytes * ATTN_TRAFFIC_PER_ALGO_BYTE),
        "traffic_source": "ncu dram bytes of a 128-row x 1055-token fused-append launch scaled by algorithmic bytes (ratio 1.014)",
        "kernel": f"cdb::decode_attn_kernel<{D},{5 if D == 96 else 4}>",
        "launch_ms": round(per_launch_ms, 4),
        "algorithmic_bytes_per_launch": int(per_launch_bytes),
        "launches_timed": n,
    }


def step_roofline(shape, recurrent_positions, coda_sizes, prefill_batches, measured_s: float, hbm_gbs: float,
                  tflops: float) -> dict:
    """Whole-step roofline: the sum over the step's launches of max(bytes / HBM bandwidth,
    FLOPs / tensor peak), against the measured step time.

    Per recurrent launch of B rows: the decode-attention bytes of every layer (kernel_bench
    attention_bytes with the append) plus the shared block's weights (2 P bytes, P = L (4 H^2 +
    3 H I) parameters), and 2 B P GEMM FLOPs. Per coda launch: the LM head's weights (2 V H bytes)
    and 2 B H V FLOPs. Per prefill batch of T prompt tokens, S recurrent steps: 2 T P S FLOPs (plus
    the LM head of its sampled rows) against the weights read once per step.
    """

    from continuous_depth_batching_b200.kernel_bench import attention_bytes

    H, I, L, V = shape.hidden_size, shape.intermediate_size, shape.num_hidden_layers, shape.vocab_size
    heads, D, S = shape.num_attention_heads, shape.head_dim, shape.total_ut_steps
    P = L * (4 * H * H + 3 * H * I)
    bw, fl = hbm_gbs * 1e9, tflops * 1e12
    parts = {"recurrent": 0.0, "coda": 0.0, "prefill": 0.0}
    for pos in recurrent_positions:
        byts = L * attention_bytes(pos, heads, D, append=True) + 2 * P
        parts["recurrent"] += max(byts / bw, 2 * len(pos) * P / fl)
    for b in coda_sizes:
        parts["coda"] += max(2 * V * H / bw, 2 * b * H * V / fl)
    for tokens, sampled in prefill_batches:
        parts["prefill"] += max((2 * P * S + 2 * V * H) / bw, (2 * tokens * P * S + 2 * sampled * H * V) / fl)
    total = sum(parts.values())
    return {
        "roofline_s": round(total, 4),
        "measured_s": round(measured_s, 4),
        "frac": round(total / measured_s, 4),
        "parts_s": {k: round(v, 4) for k, v in parts.items()},
        "hbm_gbs": hbm_gbs,
        "tflops": tflops,
        "launches": {"recurrent": len(recurrent_positions), "coda": len(coda_sizes), "prefill": len(prefill_batches)},
    }


def run_b200(args) -> None:
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        # ranks wait for one another only at the start/end barriers and the result reduction;
        # a rank that never arrives ends the others' collective with an error after this timeout
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    if args.config == 3 and args.requests == 256:
        args.requests = 128  # 128 requests
    if args.config == 2 and args.requests == 256:
        args.requests = 512  # 512 requests
    eng, shape = build_engine(args, device)
    prompts, max_new, depths, arrivals = config_workload(args, rank, world)
    stream = eng.runner.stream

    def step():
        return eng.generate_batch(prompts, max_new_tokens=max_new, eos_token_id=None, exit_depths=depths,
                                  arrival_offsets_s=arrivals)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # Record representative attention launch shapes (positions) from the workload for the roofline pass.
    recorded: list[tuple[list[int], list[int]]] = []
    rec_positions: list[list[int]] = []
    coda_sizes: list[int] = []
    prefill_batches: list[tuple[int, int]] = []
    prefill_events: list[tuple[torch.cuda.Event, torch.cuda.Event]] = []
    orig = eng._run_recurrent
    orig_coda, orig_prefill = eng._run_coda, eng._run_prefill

    def recorder(items):
        if eng.last_stats.recurrent_batches % 5 == 0:
            recorded.append(([it.req.slot for it in items], [it.position for it in items]))
        rec_positions.append([it.position for it in items])
        return orig(items)

    def coda_recorder(items):
        coda_sizes.append(len(items))
        return orig_coda(items)

    def prefill_recorder(batch):
        prefill_batches.append((sum(q for _r, _p, q, _h in batch), sum(int(h) for *_x, h in batch)))
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        out = orig_prefill(batch)
        b.record(stream)
        prefill_events.append((a, b))
        return out

    peaks_path = ROOT / "MEASURED_PEAKS.json"
    peak_gbs = json.loads(peaks_path.read_text())["hbm_gbs"] if peaks_path.exists() else 6650.0
    peak_src = "measured" if peaks_path.exists() else "fallback"
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    gen_tokens = 0
    launches0 = eng.runner.stats.kernel_launches
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        torch.cuda.nvtx.range_push("bench.timed")
        t0 = time.perf_counter()
        ev0.record(stream)
        for _ in range(args.steps):
            eng._run_recurrent, eng._run_coda, eng._run_prefill = recorder, coda_recorder, prefill_recorder
            outs = step()
            eng._run_recurrent, eng._run_coda, eng._run_prefill = orig, orig_coda, orig_prefill
            gen_tokens += sum(len(o.generated_tokens) for o in outs)
        ev1.record(stream)
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        torch.cuda.nvtx.range_pop()
    dev_s = ev0.elapsed_time(ev1) / 1e3
    wall_s = t1 - t0
    prefill_s = sum(a.elapsed_time(b) for a, b in prefill_events) / 1e3
    local_dev_s = dev_s
    kernel_launches = eng.runner.stats.kernel_launches - launches0
    stats = eng.last_stats
    decode_s, _, _ = aggregate(dev_s - prefill_s, 0.0, 0.0, device)
    dev_s, wall_s, total_tokens = aggregate(dev_s, wall_s, float(gen_tokens), device)
    if rank == 0:
        # 60 launches spread evenly over the timed steps (every 5th recurrent launch was recorded)
        sample = [recorded[int(i * len(recorded) / 60)] for i in range(60)] if len(recorded) > 60 else recorded
        roof = attention_roofline(eng, shape, sample, peak_gbs)
        roof["peak_source"] = peak_src
        peaks = json.loads(peaks_path.read_text()) if peaks_path.exists() else {}
        whole = None
        if args.config != 3:
            whole = step_roofline(
                shape, rec_positions, coda_sizes, prefill_batches, local_dev_s, peak_gbs,
                peaks.get("bf16_tflops_sustained", 1400.0),
            )
            whole["scope"] = "rank 0, all timed steps; peaks: measured HBM copy and sustained cuBLAS bf16"
        prompt_bytes = sum(len(p) for p in prompts) * 4 * 3
        line = {
            "metric": METRIC,
            "value": round(total_tokens / dev_s, 1),
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(dev_s * 1e3 / args.steps, 2),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded lognormal lengths, uniform token ids, categorical exit depths)",
            "config": {
                "workload": CONFIG_LABELS[args.config] + ("" if args.config != 2 else
                                                          (", refill off" if args.no_refill else ", refill on")),
                "requests_per_gpu": args.requests,
                "out_cap": args.out_cap,
                "generated_tokens_per_step_per_gpu": gen_tokens // max(args.steps, 1),
                "recurrent_batches": stats.recurrent_batches,
                "coda_batches": stats.coda_batches,
                "prefill_batches": stats.prefill_batches,
                "mean_recurrent_batch": round(stats.mean_recurrent_batch_size, 1),
                "exit_depth_histogram": {str(k): v for k, v in sorted(stats.exit_depth_histogram.items())},
                "l2": "inputs larger than L2 (KV cache tens of GB, weights 2.5 GB)",
                "cuda_graphs": not args.no_graph,
                "gemm": "libcdb stream-K tcgen05 (projections, fused SwiGLU, fused LM head + argmax)",
                "lm_head": args.lm_head,
                "parallelism": f"{world} independent request-sharded replicas (no collective)",
            },
            "e2e": {
                "value": round(total_tokens / wall_s, 1),
                "unit": UNIT,
                "h2d_bytes_per_step": prompt_bytes,
                "d2h_bytes_per_step": (gen_tokens // max(args.steps, 1)) * 8,
            },
            "decode_only": {
                "value": round(total_tokens / decode_s, 1),
                "unit": UNIT,
                "prefill_ms_per_step_rank0": round(prefill_s * 1e3 / args.steps, 2),
                "definition": "generated tokens / (device time minus prefill launch time), max over ranks",
            },
            "gpu_launches": kernel_launches,
            "flop_bound": flop_bound_summary(shape, stats),
            "roofline": roof,
            "step_roofline": whole,
            "clocks": clocks.summary(),
        }
        if world == 1 and not args.no_cpu_baseline and args.config == 1:
            line["same_sample"] = gpu_on_cpu_sample(eng)
            line["cpu_baseline"] = cpu_baseline(seconds=20.0)
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


CONFIG_LABELS = {
    1: "BASELINE config 1: Ouro-1.4B random-init, 256 concurrent requests, lognormal lengths, replayed categorical "
       "depths (0.2,0.3,0.3,0.2), kv single, block 16, refill on",
    2: "BASELINE config 2: Ouro-2.6B (48 layers) random-init, 512 requests, Poisson arrivals at 20 req/s, lognormal "
       "lengths, categorical depths (0.1,0.2,0.3,0.4), per-step KV as last_exited with reserve admission, block 16",
    3: "BASELINE config 3: Huginn-0125 random-init (2/4/2 blocks, 5280 wide, 55x96 heads), 128 requests, prompts "
       "U[64,512], 256 new tokens, truncated geometric depths (mean 12, 1..32), kv single, block 16, refill on",
}


def flop_bound_summary(shape, stats) -> dict:
    """The eq. (1) FLOP bound on the speed-up of this run's exit schedule over full depth
    (``continuous_depth_batching_b200.flop_bound``), from the model's stage weights (counted on a
    ``meta``-device model) and the mean recurrent steps per decoded token of the last step."""

    from continuous_depth_batching_b200 import HuginnForCausalLM, OuroForCausalLM
    from continuous_depth_batching_b200.flop_bound import stage_flops

    huginn = hasattr(shape, "n_embd")
    steps = shape.total_recurrent_steps if huginn else shape.total_ut_steps
    with torch.device("meta"):
        f = stage_flops(HuginnForCausalLM(shape) if huginn else OuroForCausalLM(shape))
    mean_depth = stats.recurrent_steps / stats.coda_tokens if stats.coda_tokens else float(steps)
    return {
        **f.to_json_dict(),
        "f0_over_fr": round(f.f0_over_fr, 4),
        "mean_recurrent_steps": round(mean_depth, 4),
        "max_depth": steps,
        "ideal_speedup_vs_full_depth": round(f.ideal_speedup(max_depth=steps, mean_depth=mean_depth), 4),
        "note": "compare with this line's value over `bench.py --engine cb` (same kernels, every token at full depth)",
    }


CPU_SAMPLE_REQUESTS = 4
CPU_SAMPLE_NEW_TOKENS = 16


def cpu_sample_workload():
    """Bounded sample of the config-1 workload for the CPU baseline: the trace's first 4 requests
    at their full prompt lengths (221, 180, 334 and 218 tokens), 16 new tokens each, the first 15
    replayed exit depths of each."""

    prompts, _max_new, depths = workload(0, 256, 1024)
    k, new = CPU_SAMPLE_REQUESTS, CPU_SAMPLE_NEW_TOKENS
    return prompts[:k], [new] * k, [d[: new - 1] for d in depths[:k]]


def sample_description() -> str:
    return (f"the first {CPU_SAMPLE_REQUESTS} config-1 requests at full prompt lengths, {CPU_SAMPLE_NEW_TOKENS} new "
            "tokens each, replayed depths (prefill included)")


def gpu_on_cpu_sample(eng, reps: int = 5) -> dict:
    """The B200 engine's tokens/s on the CPU baseline's sample (device time, CUDA events), so the
    two arms can be compared on identical work."""

    prompts, max_new, depths = cpu_sample_workload()
    stream = eng.runner.stream
    eng.generate_batch(prompts, max_new_tokens=max_new, eos_token_id=None, exit_depths=depths)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    tokens = 0
    for _ in range(reps):
        outs = eng.generate_batch(prompts, max_new_tokens=max_new, eos_token_id=None, exit_depths=depths)
        tokens += sum(len(o.generated_tokens) for o in outs)
    b.record(stream)
    b.synchronize()
    return {"value": round(tokens / (a.elapsed_time(b) / 1e3), 1), "unit": UNIT, "sample": sample_description(),
            "runs": reps}


def cpu_baseline(seconds: float = 20.0, max_runs: int = 3) -> dict:
    """Time the CPU restatement of the reference engine (oracle/) on this host's cores."""

    from continuous_depth_batching_b200.ouro import OuroShape, random_ouro_state_dict
    from oracle.engine import OracleConfig, OracleEngine

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    shape = OuroShape(**OURO_1P4B)
    sd = random_ouro_state_dict(shape, seed=1234, dtype=torch.float32)
    cfg = OracleConfig(num_blocks=1024, max_model_len=4096, synthetic_exit_replay=True, max_recurrent_steps=4)
    eng = OracleEngine(shape, sd, cfg, torch.float32)
    prompts, max_new, depths = cpu_sample_workload()
    tokens, t0 = 0, time.perf_counter()
    runs = 0
    while True:
        out = eng.generate(prompts, max_new, exit_depths=depths)
        tokens += sum(len(x) for x in out)
        runs += 1
        if time.perf_counter() - t0 > seconds or runs >= max_runs:
            break
    dt = time.perf_counter() - t0
    cpu_model = ""
    try:
        for ln in Path("/proc/cpuinfo").read_text().splitlines():
            if ln.startswith("model name"):
                cpu_model = ln.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {
        "value": round(tokens / dt, 3),
        "unit": UNIT,
        "cores": threads,
        "cpu_model": cpu_model,
        "dtype": "fp32",
        "kind": "port",
        "sample": f"{runs} x generate of {sample_description()}, fp32 on the host CPU",
    }


def run_reference(args) -> None:
    rank, world, _ = dist_env()
    if rank != 0:
        return
    t_all = []
    vals = []
    for i in range(args.warmup + args.steps):
        b = cpu_baseline(seconds=5.0, max_runs=1)
        if i >= args.warmup:
            vals.append(b["value"])
            t_all.append(b)
    v = statistics.mean(vals) if vals else 0.0
    line = {
        "metric": METRIC,
        "value": round(v, 3),
        "unit": UNIT,
        "impl": "reference",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": f"BASELINE config 1 sample: {sample_description()}"},
        "cpu_baseline": {**t_all[-1], "value": round(v, 3)} if t_all else None,
        "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_cb(args) -> None:
    """The full-depth CB baseline on one GPU: generated tokens / device time over K timed steps."""

    from continuous_depth_batching_b200 import ContinuousBatchingConfig, ContinuousBatchingEngine, OuroForCausalLM, OuroShape

    rank, world, local = dist_env()
    if world > 1:
        if rank == 0:
            print(json.dumps({"engine": "cb", "unavailable": "the CB baseline line is measured on one GPU"}))
        return
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    shape = OuroShape(**OURO_1P4B)
    model = OuroForCausalLM.random_init(shape, seed=1234, dtype=torch.bfloat16, device=device)
    cfg = ContinuousBatchingConfig(
        block_size=16, num_blocks=args.num_blocks, use_async_batching=True, use_cuda_graph=not args.no_graph,
        max_model_len=4096, max_num_seqs=256,
    )
    eng = ContinuousBatchingEngine.from_model(
        model, cfg, device=device, kv_policy="single", fused_lm_head=getattr(args, "lm_head", "fused") == "fused",
    )
    del model
    prompts, max_new, _depths = workload(replica_seed(args.seed, rank), args.requests, args.out_cap)
    stream = eng.runner.stream

    def step():
        return eng.generate_batch(prompts, max_new_tokens=max_new, eos_token_id=None)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tokens = 0
    with ClockSampler(local) as clocks:
        ev0.record(stream)
        for _ in range(args.steps):
            outs = step()
            tokens += sum(len(o.generated_tokens) for o in outs)
        ev1.record(stream)
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    st = eng.last_stats
    print(json.dumps({
        "metric": "decode tokens/s/GPU, Ouro-1.4B full-depth continuous batching (baseline engine, same kernels)",
        "engine": "cb",
        "value": round(tokens / (ms / 1e3), 1),
        "unit": UNIT,
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 2),
        "higher_is_better": True,
        "dtype": "bf16",
        "data": "synthetic (the CDB line's seeded requests; every token at full depth)",
        "config": {"workload": "BASELINE config 1 requests, full-depth CB baseline", "requests": args.requests,
                   "kv_policy": "single", "use_async_batching": True},
        "batches": {"prefill": st.prefill_batches, "decode": st.decode_batches,
                    "mean_decode_batch": round(st.mean_decode_batch_size, 1)},
        "clocks": clocks.summary(),
    }))


def run_config4(args) -> None:
    """one seeded Poisson trace shared round-robin by the ranks, one pass."""

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900), device_id=device)
    eng, _shape = build_engine(args, device)
    prompts, max_new, depths, arrivals = config4_trace(args.seed, args.trace_requests, args.rate, args.out_cap)
    mine = list(range(rank, len(prompts), world))
    p_m = [prompts[i] for i in mine]
    n_m = [max_new[i] for i in mine]
    d_m = [depths[i] for i in mine]
    a_m = [arrivals[i] for i in mine]
    # warm-up: graphs for every launch width up to 256 rows, on this rank's first requests
    k = min(256, len(p_m))
    for _ in range(max(1, args.warmup)):
        eng.generate_batch(p_m[:k], max_new_tokens=[min(8, m) for m in n_m[:k]], eos_token_id=None,
                           exit_depths=[d[: min(8, m) - 1] for d, m in zip(d_m[:k], n_m[:k], strict=True)])
    torch.cuda.synchronize()
    stream = eng.runner.stream
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        t0 = time.perf_counter()
        ev0.record(stream)
        outs = eng.generate_batch(p_m, max_new_tokens=n_m, eos_token_id=None, exit_depths=d_m, arrival_offsets_s=a_m)
        ev1.record(stream)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    dev_s = ev0.elapsed_time(ev1) / 1e3
    tokens = sum(len(o.generated_tokens) for o in outs)
    dev_max, wall_max, total = aggregate(dev_s, wall, float(tokens), device)
    if rank == 0:
        print(json.dumps({
            "metric": METRIC,
            "value": round(total / dev_max, 1),
            "unit": UNIT,
            "n_gpus": world,
            "steps": 1,
            "warmup": max(1, args.warmup),
            "ms_per_step": round(dev_max * 1e3, 2),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded lognormal lengths, uniform token ids, categorical depths, Poisson arrivals)",
            "config": {
                "workload": f"BASELINE config 4: {args.trace_requests} requests, Poisson arrivals at {args.rate} req/s "
                "total, request i on rank i mod N, Ouro-1.4B random-init, refill on",
                "last_arrival_s": round(arrivals[-1], 2),
                "parallelism": f"{world} request-sharded replicas (no collective on the hot path)",
                "tokens": int(total),
            },
            "e2e": {"value": round(total / wall_max, 1), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": int(total) * 8},
            "rank0_tokens_per_s": round(tokens / dev_s, 1),
            "clocks": clocks.summary(),
        }), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def main() -> None:
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.engine == "cb":
        run_cb(args)
    elif args.config == 4:
        run_config4(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
