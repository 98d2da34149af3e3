"""Parity of the engine exactly as ``bench.py`` builds and times it.

The model is the bench's: the Ouro-1.4B architecture (24 layers, hidden 2048, 16 x 128 heads,
SwiGLU 5632, vocab 49152, 4 recurrent steps) with the bench's seeded bf16 random init, the bench's
engine configuration (block 16, ``single`` KV, refill, synchronous replay, CUDA graphs, the fused
tcgen05 LM head + argmax) and the bench's own requests: the first six of the seeded config-1
workload at their full prompt lengths (130-334 tokens), 16 new tokens each, replaying the first
15 exit depths of each request's seeded categorical schedule.

Checks, against the CPU oracle run on the same bf16 weights:

* the launch trace (every prefill / recurrent / coda launch, each item's position, recurrent step
  and block-table row) equals the fp32 oracle's bit for bit;
* teacher-forced on the fp32 oracle's tokens, the LM-head logits meet ``tests/numerics.py`` (as
  accurate against fp32 as the reference-style bf16 evaluation, closer to it than it is to
  fp32, greedy tokens equal at >= 99% of the positions its margin decides);
* the fused LM head's greedy tokens (the path the bench times) equal the argmax of the stored
  logits at >= 99% of positions and the bf16 oracle's at >= 99% of decided positions.

The absolute max-abs logit errors are printed beside BASELINE's 2e-2 figure.
"""

from __future__ import annotations

import os
from types import SimpleNamespace

import pytest
import torch

import bench
from continuous_depth_batching_b200 import OuroShape
from continuous_depth_batching_b200.ouro import random_ouro_state_dict
from oracle.engine import OracleConfig, OracleEngine
from tests.numerics import assert_report, compare_lm_launches

pytestmark = pytest.mark.gpu

N_REQUESTS = 6
NEW_TOKENS = 16


def _requests():
    prompts, _max_new, depths = bench.workload(bench.replica_seed(0, 0), 256, 1024)
    prompts = prompts[:N_REQUESTS]
    depths = [d[: NEW_TOKENS - 1] for d in depths[:N_REQUESTS]]
    assert all(len(d) == NEW_TOKENS - 1 for d in depths)
    return prompts, [NEW_TOKENS] * N_REQUESTS, depths


def _oracle(shape, sd, prompts, max_new, depths, dtype, forced=None):
    cfg = OracleConfig(
        block_size=16, num_blocks=4096, max_recurrent_steps=shape.total_ut_steps, max_model_len=4096,
        synthetic_exit_replay=True, kv_policy="single", refill=True,
    )
    eng = OracleEngine(shape, sd, cfg, dtype)
    toks = eng.generate(prompts, max_new, exit_depths=depths, forced_tokens=forced)
    return eng, toks


def _predictions_in_token_order(eng, rows: list) -> list:
    """Per-row values of the LM-head launches (in launch order) rearranged into the order of the
    requests' generated tokens (request by request, position by position)."""

    launches = [ln for ln in eng.launch_trace if ln["kind"] in ("prefill", "coda")]
    keyed: dict[tuple[int, int], object] = {}
    i = 0
    for launch in launches:
        if launch["kind"] == "coda":
            keys = [(req, pos) for req, pos, _step in launch["items"]]
        else:
            keys = [(req, past + q - 1) for req, past, q, has in launch["items"] if has]
        for k in keys:
            keyed[k] = rows[i]
            i += 1
    assert i == len(rows)
    return [keyed[k] for k in sorted(keyed)]


def test_bench_engine_matches_oracle_at_config1():
    torch.set_num_threads(os.cpu_count() or 1)
    shape = OuroShape(**bench.OURO_1P4B)
    device = torch.device("cuda", torch.cuda.current_device())
    args = SimpleNamespace(num_blocks=4096, no_graph=False, lm_head="fused")
    eng, eshape = bench.build_engine(args, device)
    assert eshape == shape and eng.runner.fused_lm_head and eng.runner.use_cuda_graph
    # the bench's weights: the same seeded draw random_init made on this device, as fp32 on the host
    sd = {k: v.float().cpu() for k, v in random_ouro_state_dict(shape, seed=1234, dtype=torch.bfloat16, device=device).items()}
    prompts, max_new, depths = _requests()

    o32, toks = _oracle(shape, sd, prompts, max_new, depths, torch.float32)
    o16, _ = _oracle(shape, sd, prompts, max_new, depths, torch.bfloat16, forced=toks)
    del sd

    # 1. The bench path itself: fused LM head + argmax, CUDA graphs, teacher-forced.
    eng.record_trace = True
    outs = eng.generate_batch(prompts, max_new_tokens=max_new, eos_token_id=None, exit_depths=depths, forced_tokens=toks)
    eng.runner.check_status()
    assert eng.launch_trace == o32.launches == o16.launches
    fused = [t for o in outs for t in o.generated_tokens]

    # 2. The same engine keeping its logits (GEMM then argmax) for the numerics criteria.
    eng.keep_logits = True
    eng.generate_batch(prompts, max_new_tokens=max_new, eos_token_id=None, exit_depths=depths, forced_tokens=toks)
    eng.runner.check_status()
    assert eng.launch_trace == o32.launches
    gpu = [lg for _, lg in eng.lm_logits]
    ref16 = [lg for _, lg in o16.logits]
    truth = [lg for _, lg in o32.logits]
    rep = compare_lm_launches(gpu, ref16, truth)
    rep["baseline_abs_bound"] = 2e-2
    print({"config1_parity": rep})
    assert_report(rep)

    # 3. The fused argmax (what the bench times) against the stored logits and the bf16 oracle,
    # position by position.
    g = torch.cat([x.float().cpu() for x in gpu])
    r = torch.cat([x.float().cpu() for x in ref16])
    stored = _predictions_in_token_order(eng, g.argmax(-1).tolist())
    ref_pred = _predictions_in_token_order(eng, r.argmax(-1).tolist())
    top2 = r.topk(2, dim=-1).values
    decided = _predictions_in_token_order(eng, ((top2[:, 0] - top2[:, 1]) > 2 * rep["gpu_vs_ref"]).tolist())
    n = len(fused)
    assert n == len(stored) == N_REQUESTS * NEW_TOKENS
    agree_stored = sum(int(fused[i] == stored[i]) for i in range(n)) / n
    dec = [i for i in range(n) if decided[i]]
    agree_ref = sum(int(fused[i] == ref_pred[i]) for i in dec) / max(1, len(dec))
    print({"fused_vs_stored_logits": agree_stored, "fused_vs_bf16_oracle_decided": agree_ref, "decided": len(dec),
           "tokens": n})
    assert agree_stored >= 0.99
    # At this random-init scale the bf16 evaluations themselves sit far apart (the bf16 oracle is
    # ~0.8 logits from fp32 after 24 layers x 4 steps), so few or no positions are decided by a
    # margin above that noise; the bar applies to the ones that are.
    if dec:
        assert agree_ref >= 0.99
