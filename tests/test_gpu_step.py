"""Single-launch parity: one recurrent step and one prefill on identical inputs, GPU vs oracle.

Both sides start from the same KV-cache contents, block tables and hidden states. The GPU
result must be as accurate (against the fp32 oracle) as the reference-style bf16 oracle is,
and the appended K/V rows must match the bf16 oracle's to rounding.
"""

from __future__ import annotations

import pytest
import torch

from continuous_depth_batching_b200 import ContinuousDepthBatchingConfig, ContinuousDepthBatchingEngine, OuroForCausalLM, OuroShape
from continuous_depth_batching_b200.ouro import random_ouro_state_dict
from oracle.ouro_math import OracleKVCache, OuroOracle, OuroWeights
from tests.numerics import assert_as_accurate_as_reference, max_abs

pytestmark = pytest.mark.gpu

SHAPES = {
    "cfg0": OuroShape(vocab_size=1024, hidden_size=256, intermediate_size=704, num_hidden_layers=4, num_attention_heads=4,
                      num_key_value_heads=4, head_dim=64, total_ut_steps=4, max_position_embeddings=2048),
    "1p4b_w": OuroShape(vocab_size=49152, hidden_size=2048, intermediate_size=5632, num_hidden_layers=2,
                        num_attention_heads=16, num_key_value_heads=16, head_dim=128, total_ut_steps=4,
                        max_position_embeddings=2048),
}


def _setup(shape_key, graphs):
    shape = SHAPES[shape_key]
    sd = random_ouro_state_dict(shape, seed=5, gate_std=0.1)
    model = OuroForCausalLM(shape)
    model.load_state_dict(sd)
    cfg = ContinuousDepthBatchingConfig(num_blocks=256, max_recurrent_steps=4, synthetic_exit_replay=True,
                                        use_async_batching=False, max_model_len=2048, use_cuda_graph=graphs)
    eng = ContinuousDepthBatchingEngine.from_model(model, cfg, device="cuda")
    eng.runner.reset(64)

    def oracle(dtype):
        return OuroOracle(OuroWeights.from_state_dict(shape, sd, dtype),
                          OracleKVCache(shape, shape.num_hidden_layers, 256, 16, dtype))

    return shape, eng, oracle(torch.bfloat16), oracle(torch.float32)


@pytest.mark.parametrize("shape_key", ["cfg0", "1p4b_w"])
@pytest.mark.parametrize("graphs", [False, True])
def test_one_recurrent_step_matches_oracle(shape_key, graphs):
    shape, eng, o16, o32 = _setup(shape_key, graphs)
    r = eng.runner
    gen = torch.Generator().manual_seed(11)
    n = 7
    positions = [0, 5, 15, 16, 33, 100, 160]
    # Request i owns resident slot i and blocks [i*12, i*12+12).
    blocks = [list(range(i * 12, i * 12 + 12)) for i in range(n)]
    for i in range(n):
        r.pool.pool.allocate(i, i, 12)
    kv = (0.5 * torch.randn(r.pool.kv.shape, generator=gen)).to(torch.bfloat16)
    r.pool.kv.copy_(kv.to("cuda"))
    for o in (o16, o32):
        for layer in range(shape.num_hidden_layers):
            o.cache.k[layer].copy_(kv[layer, 0])
            o.cache.v[layer].copy_(kv[layer, 1])
    hidden = torch.randn(n, shape.hidden_size, generator=gen).to(torch.bfloat16)
    slots = [3 * i + 1 for i in range(n)]
    r.bank[torch.tensor(slots)] = hidden.to("cuda")
    r.recurrent(list(range(n)), positions, slots, 0, True)
    torch.cuda.synchronize()
    got = r.bank[torch.tensor(slots)].cpu()
    gate = r.gate_out[:n].cpu()
    want16, gate16 = o16.recurrent_step(hidden, positions, blocks, 0)
    want32, gate32 = o32.recurrent_step(hidden.float(), positions, blocks, 0)
    e_state = assert_as_accurate_as_reference(got, want16, want32, f"{shape_key} state")
    e_gate = assert_as_accurate_as_reference(gate, gate16, gate32, f"{shape_key} gate", floor=2e-2)
    print(f"{shape_key} graphs={graphs}: state err gpu/ref {e_state}, gate err gpu/ref {e_gate}, "
          f"gpu-vs-bf16 {max_abs(got, want16):.3e}")
    kv_gpu = r.pool.kv.cpu()
    last = shape.num_hidden_layers - 1
    for i, p in enumerate(positions):
        row = blocks[i][p // 16] * 16 + p % 16
        k16 = o16.cache.k[last][row]
        assert max_abs(kv_gpu[last, 0, row], k16) <= 2 ** -6 * max(1.0, k16.float().abs().max().item()), i


@pytest.mark.parametrize("shape_key", ["cfg0", "1p4b_w"])
def test_one_prefill_matches_oracle(shape_key):
    shape, eng, o16, o32 = _setup(shape_key, False)
    r = eng.runner
    gen = torch.Generator().manual_seed(12)
    lens = [37, 5, 64, 1]
    blocks = [list(range(i * 12, i * 12 + 12)) for i in range(len(lens))]
    for i in range(len(lens)):
        r.pool.pool.allocate(i, i, 12)
    chunks, ids, slots, pos = [], [], [], []
    for i, ln in enumerate(lens):
        toks = torch.randint(0, shape.vocab_size, (ln,), generator=gen).tolist()
        chunks.append((toks, 0, blocks[i]))
        ids += toks
        slots += [i] * ln
        pos += list(range(ln))
    ends = [int(e) for e in torch.tensor(lens).cumsum(0) - 1]
    logits = r.prefill(ids, slots, pos, ends, [0, 1, 2, 3], [0, 1, 2, 3], [0, 0, 0, 0], keep_logits=True)
    torch.cuda.synchronize()
    sel = torch.tensor(ends)
    l16 = o16.lm_head(o16.prefill(chunks, [0, 0, 0, 0])[sel])
    l32 = o32.lm_head(o32.prefill(chunks, [0, 0, 0, 0])[sel])
    errs = assert_as_accurate_as_reference(logits, l16, l32, f"{shape_key} prefill logits")
    print(f"{shape_key}: prefill logit err gpu/ref {errs}, gpu-vs-bf16 {max_abs(logits, l16):.3e}")
