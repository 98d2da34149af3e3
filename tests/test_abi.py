"""CPU checks of the C ABI boundary: the library builds, loads and exports every declared symbol.

No compute is called here (there is no GPU in the CPU suite); the GPU tests call every entry
point through the same ctypes binding.
"""

from __future__ import annotations

import re
from pathlib import Path

from continuous_depth_batching_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols() -> list[str]:
    text = (ROOT / "include" / "cdb_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(cdb_[a-z0-9_]+)\s*\(", text)))


def test_header_and_binding_agree():
    assert declared_symbols() == sorted(_lib.exported_symbols())


def test_library_loads_and_exports_every_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.cdb_version() >= 100
    assert lib.cdb_status_string(0) == b"ok"
    assert lib.cdb_status_string(4).startswith(b"device-side wait")


def test_invalid_arguments_are_rejected_without_launching():
    lib = _lib.load()
    # block_size other than 16 and unsupported head shapes fail on the host, before any launch.
    assert lib.cdb_attn_plan(None, 0, 1, 16, 128, 32, 10, 10, 148, None, None, None) == 1
    assert lib.cdb_attn_plan(None, 0, 1, 7, 128, 16, 10, 10, 148, None, None, None) == 2
    assert lib.cdb_rmsnorm(None, 0, None, None, None, 0, None, 0, 1, 100, 1e-6, None) == 1
    assert lib.cdb_silu_mul(None, 0, None, 0, 1, 7, None) == 1
    assert lib.cdb_argmax(None, 0, 1, 0, None, None, None, None, None) == 1
    assert lib.cdb_attn_scratch_bytes(256, 16, 128) > 0
