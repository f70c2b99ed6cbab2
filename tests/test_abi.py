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


def test_noalloc_decode_checks_arguments_before_touching_the_device():
    """A rejected call to the allocation-free decode attention returns its
    argument error before any CUDA call (so nothing is queued on the caller's
    stream): on a host without a GPU a bad head ratio or split still reports
    the argument error, while a valid call fails only at the device lookup."""
    lib = _lib.load()
    args = dict(q=None, out=None, k=None, v=None, nb=64, bt=None, mb=8, rows=None, seqlens=None, ctx_add=1, batch=4,
                hq=16, hkv=8, bs=256, scale=0.088, split=0, maxc=2048, stream=None)

    def call(**kw):
        a = dict(args, **kw)
        return lib.aacc_paged_decode_attention_noalloc(
            a["q"], a["out"], a["k"], a["v"], a["nb"], a["bt"], a["mb"], a["rows"], a["seqlens"], a["ctx_add"],
            a["batch"], a["hq"], a["hkv"], a["bs"], a["scale"], a["split"], a["maxc"], a["stream"])

    assert call(hq=12, hkv=4) == 3                   # AACC_ERR_UNSUPPORTED: G = 3
    assert b"head ratio" in lib.aacc_last_error()
    assert call(split=100) == 1                      # AACC_ERR_INVALID: split not a multiple of the tile
    assert call(bs=100) == 1                         # AACC_ERR_INVALID: block size
    assert call(batch=0) == 0                        # nothing to do
    import torch
    if not torch.cuda.is_available():
        assert call() == 2                           # AACC_ERR_CUDA: valid arguments reach the device lookup
