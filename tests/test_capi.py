"""The C ABI library loads and exports every entry point include/moe_b200.h
declares, and the ctypes binding covers exactly those (no GPU needed)."""

import re
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def declared():
    text = (ROOT / "include" / "moe_b200.h").read_text()
    return sorted(set(re.findall(r"^MOE_API\s+[\w\s\*]+?\b(moe_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = declared()
    assert "moe_route" in names and "moe_grouped_gemm_up" in names and len(names) >= 15


def test_library_exports_every_declared_symbol():
    import ctypes

    from moe_b200 import _lib

    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_matches_header():
    from moe_b200 import _lib

    assert sorted(_lib.EXPORTED) == declared()


def test_status_strings():
    from moe_b200 import _lib

    assert _lib.lib.moe_status_string(0) == b"ok"
    assert b"range" in _lib.lib.moe_status_string(-6)
    assert _lib.version().startswith("moe_b200")
