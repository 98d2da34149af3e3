"""torch.ops.cdb registration (CPU): every op has its schema, and CPU tensors are refused loudly
(there is no CPU path)."""

from __future__ import annotations

import pytest
import torch

import continuous_depth_batching_b200.ops  # noqa: F401  (registers torch.ops.cdb.*)

OPS = ["gemm_bf16", "mlp_gateup_silu", "lm_head_argmax", "add_rmsnorm", "paged_decode_attention", "exit_gate_route"]


@pytest.mark.parametrize("name", OPS)
def test_op_registered(name):
    schema = str(getattr(torch.ops.cdb, name).default._schema)
    assert schema.startswith(f"cdb::{name}(")


def test_cpu_tensors_refused():
    x = torch.zeros(2, 8, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        torch.ops.cdb.gemm_bf16(x, torch.zeros(4, 8, dtype=torch.bfloat16), torch.zeros(2, 4, dtype=torch.bfloat16))
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        torch.ops.cdb.lm_head_argmax(x, torch.zeros(16, 8, dtype=torch.bfloat16))
