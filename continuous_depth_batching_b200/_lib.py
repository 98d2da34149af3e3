"""ctypes binding of the C ABI in ``include/cdb_b200.h`` (``libcdb_b200.so``).

The library is the only compute path: if it is missing this module raises on first use
instead of falling back to anything else. Build it with
``python -m continuous_depth_batching_b200.csrc.build``.
"""

from __future__ import annotations

import ctypes
from ctypes import c_double, c_float, c_int, c_int64, c_void_p
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libcdb_b200.so"

# int32 entries of an attention work-plan header (CDB_ATTN_PLAN_HEADER_INTS in the C header)
ATTN_PLAN_MAX_CHUNKS = 1024
ATTN_PLAN_HEADER_INTS = 4 + ATTN_PLAN_MAX_CHUNKS + 1

# name -> argtypes (all return int status unless listed in _RESTYPES)
_SIGNATURES: dict[str, list] = {
    "cdb_version": [],
    "cdb_status_string": [c_int],
    "cdb_attn_plan": [c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p],
    "cdb_paged_decode_attn_append": [
        c_void_p, c_int64, c_int64, c_int64,  # qkv, stride, k_col, v_col
        c_void_p, c_int64,  # out, out_stride
        c_void_p, c_int, c_int64, c_int,  # kv_base, num_cache_layers, kv_rows, cache_layer
        c_void_p, c_int64, c_void_p, c_void_p,  # block_table, stride, item_slot, item_pos
        c_int, c_void_p, c_void_p, c_void_p, c_int,  # rope_mode, cos, sin, qk_bias, append
        c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,  # plan_header, units, part_o, part_ml, counters
        c_int, c_int, c_int, c_int, c_int,  # scratch_items, num_items, num_heads, head_dim, block_size
        c_float, c_int, c_void_p, c_void_p,  # scale, num_ctas, status, stream
    ],
    "cdb_paged_decode_attn_append_static": [
        c_void_p, c_int64, c_int64, c_int64,  # qkv, stride, k_col, v_col
        c_void_p, c_int64,  # out, out_stride
        c_void_p, c_int, c_int64, c_int,  # kv_base, num_cache_layers, kv_rows, cache_layer
        c_void_p, c_int64, c_void_p, c_void_p,  # block_table, stride, item_slot, item_pos
        c_int, c_void_p, c_void_p, c_void_p, c_int,  # rope_mode, cos, sin, qk_bias, append
        c_int, c_int, c_int, c_int,  # num_items, num_heads, head_dim, block_size
        c_float, c_int, c_void_p, c_void_p,  # scale, num_ctas, status, stream
    ],
    "cdb_mlp_gateup_silu_gemm": [
        c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64,  # x, ldx, w_gate_up, ldw, act, ld_act
        c_int, c_int, c_int, c_int,  # M, inter, K, max_ctas
        c_void_p, c_int64, c_void_p, c_int,  # workspace, workspace_elems, counters, num_counters
        c_int, c_void_p, c_void_p,  # num_sms, status, stream
    ],
    "cdb_attn_scratch_bytes": [c_int, c_int, c_int],
    "cdb_rope_append_kv": [
        c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int, c_int64, c_int,
        c_void_p, c_int64, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p,  # ... cos, sin, qk_bias
        c_int, c_int, c_int, c_int, c_void_p,
    ],
    "cdb_prefill_attention": [
        c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_int, c_int64, c_int,
        c_void_p, c_int64, c_void_p, c_int, c_int, c_int, c_int, c_float, c_void_p, c_void_p,
    ],
    "cdb_gemm_bf16": [
        c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_int, c_int, c_int,
        c_int, c_void_p, c_int64, c_void_p, c_int, c_int, c_void_p, c_void_p,
    ],
    "cdb_gemm_workspace_elems": [c_int, c_int, c_int, c_int],
    "cdb_gemm_counter_elems": [c_int, c_int, c_int],
    "cdb_gemm_bf16_partials": [
        c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
    ],
    "cdb_gemm_partial_splits": [c_int, c_int, c_int, c_int],
    "cdb_lm_head_argmax": [
        c_void_p, c_int64, c_void_p, c_int64, c_int, c_int, c_int,  # x, ldx, w, ldw, M, vocab, K
        c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,  # out_ids, out_rows, token_rows, table, keys, done
        c_void_p, c_int64, c_void_p, c_int,  # workspace, workspace_elems, counters, num_counters
        c_int, c_void_p, c_void_p,  # num_sms, status, stream
    ],
    "cdb_rmsnorm": [
        c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_int64, c_int, c_int, c_float, c_void_p,
    ],
    "cdb_add_rmsnorm": [
        c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int64, c_void_p,
        c_void_p, c_void_p, c_void_p, c_int, c_int, c_float, c_void_p,
    ],
    "cdb_add_rmsnorm_parts": [
        c_void_p, c_int64, c_void_p, c_int, c_int64, c_void_p, c_void_p, c_void_p, c_int64, c_void_p,
        c_void_p, c_void_p, c_void_p, c_int, c_int, c_float, c_void_p,
    ],
    "cdb_silu_mul": [c_void_p, c_int64, c_void_p, c_int64, c_int, c_int, c_void_p],
    "cdb_gather_rows": [c_void_p, c_int64, c_void_p, c_int, c_int, c_void_p, c_int64, c_void_p],
    "cdb_argmax": [c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p],
    "cdb_embed": [
        c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_int, c_float, c_void_p,
        c_void_p,
    ],
    "cdb_sandwich_norm": [
        c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_void_p,
        c_void_p, c_int64, c_int, c_int, c_float, c_void_p,
    ],
    "cdb_latent_diff": [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int, c_int, c_void_p, c_void_p],
    "cdb_block_table_update": [c_void_p, c_int64, c_void_p, c_int, c_void_p],
    "cdb_exit_kv_copy": [c_void_p, c_int, c_int64, c_int, c_int, c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p],
    "cdb_kv_blocks_host_copy": [
        c_void_p, c_int, c_int64, c_int64, c_int, c_int, c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_void_p,
    ],
    "cdb_exit_hazard": [
        c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_double, c_void_p,
    ],
    "cdb_exit_gate_route": [
        c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
        c_int, c_int, c_double, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
    ],
    "cdb_qkv_rope_append_gemm": [
        c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int64, c_int, c_int, c_void_p, c_int,
        c_int64, c_int, c_void_p, c_int64, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int,
        c_int, c_void_p, c_int64, c_void_p, c_int, c_int, c_void_p, c_void_p,
    ],
    "cdb_o_proj_residual_norm_gemm": [
        c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
        c_int64, c_int, c_int, c_int, c_float, c_void_p, c_int64, c_void_p, c_int, c_int, c_void_p, c_void_p,
    ],
    "cdb_down_residual_norm_gemm": [
        c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
        c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_float, c_void_p, c_int64, c_void_p,
        c_int, c_int, c_void_p, c_void_p,
    ],
    "cdb_schedule_tick": [
        c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_int,
        c_int, c_int, c_int, c_void_p, c_void_p,
    ],
    "cdb_schedule_queues_init": [c_void_p, c_int, c_void_p],
    "cdb_block_pool_init": [c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p],
    "cdb_block_alloc": [
        c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p, c_void_p, c_int, c_void_p, c_void_p,
    ],
    "cdb_block_free": [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_int, c_void_p],
    "cdb_build_tables": [
        c_void_p, c_int64, c_void_p, c_int, c_int, c_void_p, c_void_p, c_int, c_int, c_void_p, c_int64, c_void_p,
        c_void_p, c_void_p, c_void_p,
    ],
}
_RESTYPES = {"cdb_status_string": ctypes.c_char_p, "cdb_attn_scratch_bytes": c_int64, "cdb_gemm_workspace_elems": c_int64,
              "cdb_gemm_counter_elems": c_int}

_LIB: ctypes.CDLL | None = None


class CDBError(RuntimeError):
    """A non-zero status from the CUDA library."""


def load() -> ctypes.CDLL:
    """Load the library once and declare every exported symbol's signature."""

    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise CDBError(
            f"{LIB_PATH} is missing: build it with `python -m continuous_depth_batching_b200.csrc.build` "
            "(the CUDA library is the only compute path; there is no fallback)"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, args in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPES.get(name, c_int)
    _LIB = lib
    return lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().cdb_status_string(rc).decode()
        raise CDBError(f"{what} failed: {msg} (status {rc})")


def ptr(t: torch.Tensor | None) -> int | None:
    """Device address of a tensor (None passes NULL)."""

    return None if t is None else t.data_ptr()


def stream_ptr(stream: torch.cuda.Stream | None = None) -> int:
    s = torch.cuda.current_stream() if stream is None else stream
    return s.cuda_stream


_NO_LAUNCH = {
    "cdb_version", "cdb_status_string", "cdb_attn_scratch_bytes", "cdb_gemm_workspace_elems", "cdb_gemm_counter_elems",
    "cdb_gemm_partial_splits",
    "cdb_schedule_queues_init",
    "cdb_kv_blocks_host_copy",
}
# Kernels enqueued through this binding (device work only; graph replays are counted by the runner).
launch_count = 0


def call(name: str, *args) -> None:
    global launch_count
    check(getattr(load(), name)(*args), name)
    if name not in _NO_LAUNCH:
        launch_count += 1


class GemmWorkspace:
    """Split-partial workspace and tile counters of the stream-K GEMM entry points
    (``cdb_gemm_bf16``, ``cdb_mlp_gateup_silu_gemm``, ``cdb_lm_head_argmax``), sized for every
    problem of up to ``max_tokens`` token rows and ``max_n`` output columns on ``num_sms`` CTAs.
    Calls sharing one workspace must be ordered (one stream); the counters stay zeroed between
    calls."""

    def __init__(self, device: torch.device, max_tokens: int, max_n: int, num_sms: int) -> None:
        bn = 256
        tile_rows = 256 if max_tokens > 256 else 128  # weight rows of one tile: 256 for prefill shapes
        self.ws = torch.zeros(2 * num_sms * tile_rows * bn, dtype=torch.float32, device=device)
        tiles = -(-max_n // 128) * max(1, -(-max_tokens // bn))
        self.ctr = torch.zeros(tiles, dtype=torch.int32, device=device)

    def args(self) -> tuple:
        """(workspace, workspace_elems, counters, num_counters) as the entry points take them."""

        return ptr(self.ws), self.ws.numel(), ptr(self.ctr), self.ctr.numel()
