"""The C-ABI library loads and exports every function the headers in include/ declare (CPU only:
no compute is launched)."""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(ROOT, "diolkos_b200", "libdiolkos.so")


def declared_functions(header: str) -> list[str]:
    src = open(header).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    src = re.sub(r"//[^\n]*", "", src)
    names = []
    for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b([A-Za-z_]\w*)\s*\(([^;{]*)\)\s*;", src, flags=re.M):
        name = m.group(1)
        if name in ("if", "for", "while", "return", "sizeof", "typedef"):
            continue
        names.append(name)
    return names


def exported_symbols(lib: str) -> set[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", lib], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


@pytest.fixture(scope="module")
def lib_symbols():
    if not os.path.exists(LIB):
        pytest.fail(f"{LIB} is not built (python -m diolkos_b200.build)")
    return exported_symbols(LIB)


HEADERS = sorted(f for f in os.listdir(INCLUDE) if f.endswith(".h"))


@pytest.mark.parametrize("header", HEADERS)
def test_header_functions_are_exported(lib_symbols, header):
    names = declared_functions(os.path.join(INCLUDE, header))
    assert names, header
    missing = [n for n in names if n not in lib_symbols]
    assert not missing, f"{header}: not exported: {missing}"


def test_library_loads_via_ctypes():
    from diolkos_b200 import _native

    L = _native.lib()
    for name in _native.SIGNATURES:
        assert hasattr(L, name)
    assert L.dk_q8_row_bytes(4096) == 4608
    assert L.dk_q8_row_bytes(288) == 336
    assert L.dk_q8_row_bytes(11008) == 12384
    assert L.dk_q8_row_bytes(100) == 0
