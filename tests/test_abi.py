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


def test_plan_header_size_matches_binding():
    text = (ROOT / "include" / "cdb_b200.h").read_text()
    chunks = int(re.search(r"#define CDB_ATTN_PLAN_MAX_CHUNKS (\d+)", text).group(1))
    assert chunks == _lib.ATTN_PLAN_MAX_CHUNKS
    assert "#define CDB_ATTN_PLAN_HEADER_INTS (4 + CDB_ATTN_PLAN_MAX_CHUNKS + 1)" in text
    assert _lib.ATTN_PLAN_HEADER_INTS == 4 + chunks + 1


def _param_kind(decl: str) -> str:
    decl = decl.strip()
    if "*" in decl:
        return "ptr"
    for kind in ("int64_t", "double", "float", "int"):
        if re.search(rf"\b{kind}\b", decl):
            return kind
    raise AssertionError(f"unrecognised parameter {decl!r}")


def test_binding_argument_kinds_match_header_prototypes():
    """Each ctypes argtype has the kind (pointer / int / int64 / float / double) of the header
    parameter in the same position, so a binding cannot shift or retype an argument."""

    import ctypes

    text = (ROOT / "include" / "cdb_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    kinds = {ctypes.c_void_p: "ptr", ctypes.c_int: "int", ctypes.c_int64: "int64_t", ctypes.c_float: "float",
             ctypes.c_double: "double"}
    protos = re.findall(r"\b(cdb_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text)
    assert len(protos) == len(_lib.exported_symbols())
    for name, params in protos:
        params = params.strip()
        header = [] if params in ("", "void") else [_param_kind(p) for p in params.split(",")]
        binding = [kinds[t] for t in _lib._SIGNATURES[name]]
        assert header == binding, (name, header, binding)


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
