"""The C-ABI library loads (no GPU needed) and exports every entry point the
header declares, and the ctypes table matches the header."""
import ctypes
import os
import re

from awesome_acceleration_b200 import _lib
from awesome_acceleration_b200.build import LIB, build

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "aacc_b200.h")


def header_functions() -> list[str]:
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return re.findall(r"\b(aacc_\w+)\s*\(", src)


def test_library_builds_and_exports_header_symbols():
    build()
    assert os.path.exists(LIB)
    lib = ctypes.CDLL(LIB)
    names = header_functions()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), f"{n} declared in aacc_b200.h but not exported"


def test_ctypes_table_matches_header():
    names = set(header_functions())
    assert names == set(_lib.SIGNATURES), names.symmetric_difference(set(_lib.SIGNATURES))
    src = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    for name, (_, args) in _lib.SIGNATURES.items():
        decl = re.search(name + r"\s*\(([^)]*)\)", src).group(1).strip()
        n_args = 0 if decl in ("void", "") else decl.count(",") + 1
        assert n_args == len(args), f"{name}: header has {n_args} args, ctypes {len(args)}"


def test_library_loads_without_gpu():
    lib = _lib.load()
    assert lib.aacc_version() >= 1
    assert _lib.load().aacc_last_error() is not None
