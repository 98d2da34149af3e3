"""The per-stage FLOP weights and the eq. (1) speed-up bound against the reference's values.

``tests/golden/flop_bound_cases.json`` holds the reference ``stage_flops`` of its own models at four
shapes (``tests/golden/make_flop_bound_cases.py``); this package's models of the same shapes,
built on the ``meta`` device, must give the same weights.
"""

from __future__ import annotations

import json
from pathlib import Path

import pytest
import torch

from continuous_depth_batching_b200.flop_bound import StageFlops, stage_flops, stage_flops_from_json
from continuous_depth_batching_b200.huginn import HuginnForCausalLM, HuginnShape
from continuous_depth_batching_b200.ouro import OuroForCausalLM, OuroShape

CASES = json.loads((Path(__file__).resolve().parent / "golden" / "flop_bound_cases.json").read_text())["cases"]


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_stage_flops_match_reference(case):
    with torch.device("meta"):
        if case["family"] == "ouro":
            model = OuroForCausalLM(OuroShape(**case["shape"]))
        else:
            model = HuginnForCausalLM(HuginnShape(**case["shape"]))
    f = stage_flops(model)
    assert (f.f0, f.fr) == (case["f0"], case["fr"])
    assert stage_flops_from_json(f.to_json_dict()) == f


def test_ideal_speedup():
    f = StageFlops(f0=1, fr=4)
    assert f.f0_over_fr == 0.25
    assert f.ideal_speedup(max_depth=4, mean_depth=2.0) == pytest.approx(17 / 9)
    assert StageFlops(f0=0, fr=3).ideal_speedup(max_depth=4, mean_depth=2.5) == pytest.approx(4 / 2.5)
    with pytest.raises(ValueError):
        f.ideal_speedup(max_depth=4, mean_depth=0)
    with pytest.raises(ValueError):
        StageFlops(f0=1, fr=0)
    with pytest.raises(TypeError):
        stage_flops(torch.nn.Linear(2, 2))


def test_bench_flop_bound_summary():
    """The bench line's ``flop_bound`` object for the Ouro-1.4B shape and a run whose decoded
    tokens took 2.5 recurrent steps on average."""

    from types import SimpleNamespace

    import bench

    case = next(c for c in CASES if c["name"] == "ouro_1p4b")
    out = bench.flop_bound_summary(OuroShape(**bench.OURO_1P4B), SimpleNamespace(recurrent_steps=250, coda_tokens=100))
    assert (out["f0_params"], out["fr_params"]) == (case["f0"], case["fr"])
    f0, fr = case["f0"], case["fr"]
    assert out["ideal_speedup_vs_full_depth"] == pytest.approx((f0 + 4 * fr) / (f0 + 2.5 * fr), abs=1e-4)
    assert out["mean_recurrent_steps"] == 2.5
