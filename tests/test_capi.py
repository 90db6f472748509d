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
    """ctypes kind of a C parameter declaration: pointer, int64, uint64 or int."""
    if "*" in param:
        return "P"
    words = param.replace("const", " ").split()
    if words[0] in ("int64_t", "long"):
        return "L"
    if words[0] == "uint64_t":
        return "U"
    if words[0] in ("int", "unsigned"):
        return "I"
    raise AssertionError(f"unmapped parameter type: {param!r}")


def test_binding_argument_types_match_prototypes():
    """Every ctypes argtypes list has the header prototype's arity and, position
    by position, its width: a pointer, a 64-bit or a 32-bit integer."""
    import ctypes

    from moe_b200 import _lib

    kinds = {ctypes.c_void_p: "P", ctypes.c_int64: "L", ctypes.c_int: "I", ctypes.c_uint64: "U"}
    protos = prototypes()
    assert sorted(protos) == declared()
    for name, (ret, params) in protos.items():
        want = [_kind(p) for p in params]
        got = [kinds[t] for t in _lib._SIGS[name]]
        assert got == want, (name, got, want)
        if ret.startswith("int64_t"):
            assert _lib._RESTYPE.get(name) is ctypes.c_int64, name
        elif ret.startswith("uint64_t"):
            assert _lib._RESTYPE.get(name) is ctypes.c_uint64, name
        elif "char" in ret:
            assert _lib._RESTYPE.get(name) is ctypes.c_char_p, name
        else:
            assert ret == "int" and name not in _lib._RESTYPE, (name, ret)


def test_header_is_plain_c_and_links(tmp_path):
    """include/moe_b200.h compiles as C99 (no C++ or torch types), and a C program
    taking the address of every declared entry point links against the library."""
    import shutil
    import subprocess

    from moe_b200 import _lib

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        import pytest

        pytest.skip("no C compiler")
    names = declared()
    src = tmp_path / "use_header.c"
    src.write_text(
        '#include "moe_b200.h"\n#include <stdio.h>\n'
        "typedef void (*fn_t)(void);\n"
        "int main(void) {\n  const fn_t fns[] = {\n"
        + "".join(f"    (fn_t)&{n},\n" for n in names)
        + "  };\n  printf(\"%d %s\\n\", (int)(sizeof(fns) / sizeof(fns[0])), moe_version());\n"
        "  return 0;\n}\n")
    exe = tmp_path / "use_header"
    lib = Path(_lib.LIB_PATH)
    r = subprocess.run([cc, "-std=c99", "-Wall", "-Werror", "-pedantic", "-I", str(ROOT / "include"),
                        str(src), "-o", str(exe), "-L", str(lib.parent), "-l:" + lib.name,
                        "-Wl,-rpath," + str(lib.parent)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, run.stderr[-2000:]
    count, version = run.stdout.split(maxsplit=1)
    assert int(count) == len(names) and version.startswith("moe_b200")
