"""CPU checks of the attention seam module: it registers under the reference's registry key and
refuses what its kernels do not serve before touching a device."""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from continuous_depth_batching_b200 import hf_attention


def test_register_installs_the_hook_under_the_reference_key():
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    before = ALL_ATTENTION_FUNCTIONS.get(hf_attention.ATTENTION_KEY)
    try:
        hf_attention.register()
        assert ALL_ATTENTION_FUNCTIONS[hf_attention.ATTENTION_KEY] is hf_attention.paged_attention_forward
    finally:
        if before is not None:
            ALL_ATTENTION_FUNCTIONS[hf_attention.ATTENTION_KEY] = before


def _cache(block_size=16):
    return SimpleNamespace(block_size=block_size, layer_index_to_group_indices={0: (0, 0)}, sliding_windows={0: 1})


@pytest.mark.parametrize("heads_kv,block,msg", [(2, 16, "MHA"), (4, 32, "block size")])
def test_unserved_shapes_raise(heads_kv, block, msg):
    q = torch.zeros(1, 4, 3, 64, dtype=torch.bfloat16)
    k = torch.zeros(1, heads_kv, 3, 64, dtype=torch.bfloat16)
    module = SimpleNamespace(layer_idx=0, scaling=0.125)
    with pytest.raises(NotImplementedError, match=msg):
        hf_attention.paged_attention_forward(module, q, k, k, None, _cache(block), None, None, 1, 1, None)


def test_cpu_cache_is_not_bound():
    cache = SimpleNamespace(key_cache=[torch.zeros(32, 4, 64, dtype=torch.bfloat16)],
                            value_cache=[torch.zeros(32, 4, 64, dtype=torch.bfloat16)])
    with pytest.raises(NotImplementedError, match="CUDA"):
        hf_attention.bind_paged_cache(cache)
