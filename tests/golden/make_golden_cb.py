"""Record the reference's full-depth continuous-batching (CB) engine on CPU.

Run in a container that has the reference checkout (read-only), with ``CDB_REFERENCE_SRC``
pointing at its ``src`` directory::

    CDB_REFERENCE_SRC=<reference checkout>/src python tests/golden/make_golden_cb.py

The reference's ``ContinuousBatchingEngine`` (``continuous_batching/continuous_api.py:133``) serves
every token at the model's full recurrent depth. It is the baseline against which CDB's speed-up
is quoted. Each tick runs either a prefill batch (whole or chunked prompts) or a decode batch (one
token per decoding request). This script drives it over BASELINE config 0's model (the weights
and CPU attention restatement of ``make_golden.py``, kv_policy ``single``) and workload in its
default pipelined mode (``use_async_batching=True``: batch k+1 is scheduled before batch k's
tokens are consumed) and in its serialized mode, with an ample cache and with KV pools too small for
the workload (recompute preemption), and with requests ending early on EOS ids or stop sequences
(pipelined, the finish is seen one tick late and the extra token computed meanwhile is dropped),
and under ``kv_pressure_mode="offload"`` with host pools of 64, 3 and 2 blocks (a victim's blocks go to
the host pool when they fit there and come back before it is scheduled again; otherwise recompute),
under ``"reserve"`` admission at 40 blocks (``max_model_len`` 512), and with a 48-token prefill budget
that chunks the prompts.
Every launched batch is recorded in order: its kind, each
request's (index, cached length, query length, samples-a-token flag) and block-table row, plus
the logits of the LM-head rows. Output: ``tests/golden/ouro_cfg0_cb.json`` and
``ouro_cfg0_cb_logits.npz``.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

import make_golden as mg  # noqa: E402  (sets up the reference import path and attention restatement)


class CBRecorder:
    """Logs every batch the reference CB engine launches, in launch order."""

    def __init__(self, engine) -> None:
        self.launches: list[dict] = []
        self.logits: list[np.ndarray] = []
        io = engine.inputs_and_outputs
        cache = engine.cache
        bs = cache.block_size
        rid_index = lambda rid: int(rid.split("-")[1])  # noqa: E731
        from looped_cdb.continuous_batching.requests import RequestStatus

        orig_prepare = io.prepare_batch_tensors

        def prepare_batch_tensors(*, requests_in_batch, **kw):
            decode = all(f.query_length == 1 and f.state.status == RequestStatus.DECODING for f in requests_in_batch)
            items = [
                [rid_index(f.state.request_id), f.state.position_offset, f.query_length, int(f.has_new_token)]
                for f in requests_in_batch
            ]
            blocks = []
            for f in requests_in_batch:
                table = cache.cache_allocator.block_table[f.state.request_id]
                n = -(-(f.state.position_offset + f.query_length) // bs)
                blocks.append([int(b) for b in table[:n]])
            self.launches.append({"kind": "decode" if decode else "prefill", "items": items, "blocks": blocks})
            return orig_prepare(requests_in_batch=requests_in_batch, **kw)

        io.prepare_batch_tensors = prepare_batch_tensors
        lm_head = engine.model.lm_head
        orig_fwd = lm_head.forward

        def lm_forward(x):
            y = orig_fwd(x)
            self.logits.append(y.detach().reshape(-1, y.shape[-1]).float().numpy().copy())
            return y

        lm_head.forward = lm_forward


def run_case(name: str, *, async_mode: bool, num_blocks: int = 4096, eos_token_id=None, stop_sequences=None,
             host_blocks: int = 0, reserve: bool = False, max_num_batched_tokens: int = 8192):
    from looped_cdb.continuous_batching.config import ContinuousBatchingConfig
    from looped_cdb.continuous_batching.continuous_api import ContinuousBatchingEngine

    model = mg.build_reference_model(mg.CFG0, "single")
    prompts, max_new = mg.config0_workload()
    cfg = ContinuousBatchingConfig(
        block_size=16,
        num_blocks=num_blocks,
        use_async_batching=async_mode,
        use_cuda_graph=False,
        use_cuda_graph_prefill=False,
        kv_pressure_mode="offload" if host_blocks else ("reserve" if reserve else "recompute"),
        # host pool of `host_blocks` blocks: one block is every cache layer's K and V rows, fp32 here
        cpu_offload_space=host_blocks * 2 * mg.CFG0.num_hidden_layers * 16 * mg.CFG0.num_key_value_heads
        * mg.CFG0.head_dim * 4 / 1024**3 if host_blocks else None,
        max_model_len=512 if reserve else 2048,
        max_num_batched_tokens=max_num_batched_tokens,
    )
    engine = ContinuousBatchingEngine.from_model(model, cfg)
    rec = CBRecorder(engine)
    with torch.no_grad():
        outs = engine.generate_batch(
            prompts, max_new_tokens=max_new, eos_token_id=eos_token_id, stop_sequences=stop_sequences, warmup=False
        )
    st = engine.last_stats
    result = {
        "name": name,
        "async": async_mode,
        "num_blocks": num_blocks,
        "num_cpu_blocks": host_blocks,
        "kv_pressure_mode": cfg.kv_pressure_mode,
        "max_model_len": cfg.max_model_len,
        "max_num_batched_tokens": cfg.max_num_batched_tokens,
        "eos_token_id": eos_token_id,
        "stop_sequences": stop_sequences,
        "tokens": [o.generated_tokens for o in outs],
        "stats": {
            "prefill_batches": st.prefill_batches,
            "prefill_requests": st.prefill_requests,
            "prefill_query_tokens": st.prefill_query_tokens,
            "decode_batches": st.decode_batches,
            "decode_tokens": st.decode_tokens,
            "recompute_preemptions": engine.offloading_manager.num_recompute_preemptions,
            "offload_preemptions": engine.offloading_manager.num_offload_preemptions,
            "restores": engine.offloading_manager.num_restores,
            "num_cpu_blocks": engine.offloading_manager._num_cpu_blocks,
        },
        "launches": rec.launches,
    }
    return result, rec.logits


def huginn_main() -> None:
    """``--huginn``: the small Huginn shape of ``make_golden_huginn.py`` (prelude, recurrent core and
    coda with their own cache layers; 6 recurrent steps; the model names no KV layout, so the
    reference cache gives every step its own slot) through the reference CB engine, pipelined and
    serialized, into ``huginn_small_cb.json``."""

    import make_golden_huginn as mh

    from looped_cdb.continuous_batching.config import ContinuousBatchingConfig
    from looped_cdb.continuous_batching.continuous_api import ContinuousBatchingEngine

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    runs = []
    for name, async_mode in (("cb_async", True), ("cb_sync", False)):
        model = mh.build_reference_model(mh.SMALL)
        prompts, max_new = mh.config0_workload()
        cfg = ContinuousBatchingConfig(
            block_size=16, num_blocks=4096, use_async_batching=async_mode, use_cuda_graph=False,
            use_cuda_graph_prefill=False, kv_pressure_mode="recompute", max_model_len=2048,
        )
        engine = ContinuousBatchingEngine.from_model(model, cfg)
        rec = CBRecorder(engine)
        with torch.no_grad():
            outs = engine.generate_batch(prompts, max_new_tokens=max_new, eos_token_id=None, warmup=False)
        st = engine.last_stats
        runs.append({
            "name": name, "async": async_mode, "num_blocks": 4096, "num_cpu_blocks": 0, "eos_token_id": None,
            "stop_sequences": None, "kv_policy": engine.cache.kv_policy,
            "tokens": [o.generated_tokens for o in outs],
            "stats": {"prefill_batches": st.prefill_batches, "prefill_requests": st.prefill_requests,
                      "prefill_query_tokens": st.prefill_query_tokens, "decode_batches": st.decode_batches,
                      "decode_tokens": st.decode_tokens, "recompute_preemptions": 0},
            "launches": rec.launches,
        })
        print(name, runs[-1]["kv_policy"], runs[-1]["stats"], flush=True)
    prompts, max_new = mh.config0_workload()
    payload = {
        "generator": "tests/golden/make_golden_cb.py --huginn",
        "shape": mh.SMALL.__dict__,
        "embed_std": mh.EMBED_STD,
        "weights_seed": 0,
        "prompts": prompts,
        "max_new_tokens": max_new,
        "block_size": 16,
        "runs": runs,
    }
    (HERE / "huginn_small_cb.json").write_text(json.dumps(payload, separators=(",", ":")))


def main() -> None:
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    runs, logits_out = [], {}
    # EOS ids 1009 and 23 and stop sequences [657, 657] and [475, 475] occur mid-generation in the
    # seeded model's full-depth output, so several requests end early
    finish = {"eos_token_id": [1009, 23], "stop_sequences": [[657, 657], [475, 475]]}
    for name, async_mode, nb, kw in (
        ("cb_async", True, 4096, {}),
        ("cb_sync", False, 4096, {}),
        ("cb_async_blocks40", True, 40, {}),
        ("cb_sync_blocks48", False, 48, {}),
        ("cb_async_eos_stop", True, 4096, finish),
        ("cb_sync_eos_stop", False, 4096, finish),
        ("cb_async_blocks40_host64", True, 40, {"host_blocks": 64}),
        ("cb_sync_blocks48_host2", False, 48, {"host_blocks": 2}),
        ("cb_async_blocks36_host3", True, 36, {"host_blocks": 3}),
        ("cb_async_reserve_blocks40", True, 40, {"reserve": True}),
        ("cb_sync_reserve_blocks40", False, 40, {"reserve": True}),
        ("cb_async_chunked48", True, 4096, {"max_num_batched_tokens": 48}),
        ("cb_sync_chunked48", False, 4096, {"max_num_batched_tokens": 48}),
    ):
        res, logits = run_case(name, async_mode=async_mode, num_blocks=nb, **kw)
        runs.append(res)
        print(name, res["stats"], len(res["launches"]), "launches", flush=True)
        if name == "cb_async":
            for i, lg in enumerate(logits):
                logits_out[f"{name}_{i}"] = lg
    prompts, max_new = mg.config0_workload()
    payload = {
        "generator": "tests/golden/make_golden_cb.py",
        "shape": mg.CFG0.__dict__,
        "gate_std": mg.GATE_STD,
        "weights_seed": 0,
        "prompts": prompts,
        "max_new_tokens": max_new,
        "block_size": 16,
        "runs": runs,
    }
    (HERE / "ouro_cfg0_cb.json").write_text(json.dumps(payload, separators=(",", ":")))
    np.savez_compressed(HERE / "ouro_cfg0_cb_logits.npz", **logits_out)


if __name__ == "__main__":
    if "--huginn" in sys.argv[1:]:
        huginn_main()
    else:
        main()
