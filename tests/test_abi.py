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


def test_small_batch_gemm_and_prefill_attention_validate_arguments_on_the_host():
    """The small-batch GEMMs and the prefill attention reject shapes they do
    not take with AACC_ERR_INVALID before any CUDA call (so this runs without
    a GPU), and a batch of zero rows is a no-op."""
    lib = _lib.load()
    sk = lib.aacc_gemm_skinny_splitk
    assert sk(None, None, None, 65, 1024, 1024, 1, None) == 1     # more than 64 rows
    assert b"M <= 64" in lib.aacc_last_error()
    assert sk(None, None, None, 4, 1000, 1024, 1, None) == 1      # N not a multiple of 128
    assert sk(None, None, None, 4, 1024, 1000, 1, None) == 1      # K not a multiple of 64
    assert sk(None, None, None, 4, 1024, 1024, 3, None) == 1      # 3 does not divide 16 slabs
    assert sk(None, None, None, 0, 1024, 1024, 4, None) == 0      # no rows
    silu = lib.aacc_skinny_silu_mul
    assert silu(None, None, None, 1, None, None, 4, 3072, 1024, None) == 1  # no counters
    pa = lib.aacc_prefill_attention
    common = (None, None, 64, None, 8, None, None, None)  # k, v, blocks, tables, max_blocks, rows, cu_q, ctx
    assert pa(None, None, 100, *common, 2, 200, 16, 8, 256, 0.088, None) == 1  # max_q_len > num_tokens
    assert pa(None, None, 100, *common, 2, 50, 16, 6, 256, 0.088, None) == 1   # 16 heads over 6 kv heads
    assert pa(None, None, 100, *common, 2, 50, 16, 8, 100, 0.088, None) == 1   # block size not a multiple of 64
