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


def prototypes():
    """name -> (return type text, [parameter type texts]) for every MOE_API function."""
    text = (ROOT / "include" / "moe_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    out = {}
    for m in re.finditer(r"MOE_API\s+([\w\s\*]+?)\b(moe_\w+)\s*\(([^)]*)\)\s*;", text):
        params = [p.strip() for p in m.group(3).split(",") if p.strip() and p.strip() != "void"]
        out[m.group(2)] = (m.group(1).strip(), params)
    return out


def _kind(param: str) -> str:
    """ctypes kind of a C parameter declaration: pointer, int64 or int."""
    if "*" in param:
        return "P"
    words = param.replace("const", " ").split()
    if words[0] in ("int64_t", "long"):
        return "L"
    if words[0] in ("int", "unsigned"):
        return "I"
    raise AssertionError(f"unmapped parameter type: {param!r}")


def test_binding_argument_types_match_prototypes():
    """Every ctypes argtypes list has the header prototype's arity and, position
    by position, its width: a pointer, a 64-bit or a 32-bit integer."""
    import ctypes

    from moe_b200 import _lib

    kinds = {ctypes.c_void_p: "P", ctypes.c_int64: "L", ctypes.c_int: "I"}
    protos = prototypes()
    assert sorted(protos) == declared()
    for name, (ret, params) in protos.items():
        want = [_kind(p) for p in params]
        got = [kinds[t] for t in _lib._SIGS[name]]
        assert got == want, (name, got, want)
        if ret.startswith("int64_t"):
            assert _lib._RESTYPE.get(name) is ctypes.c_int64, name
        elif "char" in ret:
            assert _lib._RESTYPE.get(name) is ctypes.c_char_p, name
        else:
            assert ret == "int" and name not in _lib._RESTYPE, (name, ret)
