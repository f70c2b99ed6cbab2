"""ctypes binding of the C ABI in ``include/aacc_b200.h`` (libaacc_b200.so).

The library is built in-tree by ``awesome_acceleration_b200.build``.  There
is no fallback: if the library is missing or fails to load, every op raises.
A non-zero status from an entry point becomes ``RuntimeError`` carrying
``aacc_last_error()``, the reference's error style (llm_tp.py:362-369).
"""
from __future__ import annotations

import ctypes
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libaacc_b200.so")

P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int
F32 = ctypes.c_float

# name -> (restype, argtypes); must match include/aacc_b200.h.
SIGNATURES: dict[str, tuple] = {
    "aacc_version": (I32, []),
    "aacc_last_error": (ctypes.c_char_p, []),
    "aacc_launch_count": (ctypes.c_ulonglong, []),
    "aacc_get_device_error": (I32, [P]),
    "aacc_get_device_error_async": (I32, [P, P]),
    "aacc_clear_device_error": (I32, []),
    "aacc_kv_store": (I32, [P, P, I64, I64, I64, P, P, P, I64, I32, I32, P]),
    "aacc_decode_slot_mapping": (I32, [P, P, P, I64, I32, I64, P, I64, P]),
    "aacc_advance_seqlens": (I32, [P, P, P, I64, P]),
    "aacc_gather_rows": (I32, [P, I64, I64, P, I64, P, P]),
    "aacc_paged_decode_workspace_bytes": (I64, [I64, I32, I64, I32]),
    "aacc_paged_decode_attention": (I32, [P, P, P, P, I64, P, I64, P, P, I32, I64, I32, I32, I32, F32, I32, I64,
                                          P, I64, P]),
    "aacc_paged_decode_attention_noalloc": (I32, [P, P, P, P, I64, P, I64, P, P, I32, I64, I32, I32, I32, F32, I32,
                                                  I64, P]),
    "aacc_paged_decode_noalloc_capacity_bytes": (I64, []),
    "aacc_prefill_attention": (I32, [P, P, I64, P, P, I64, P, I64, P, P, P, I64, I64, I32, I32, I32, F32, P]),
    "aacc_prefill_attention_mma": (I32, [P, P, P, P, I64, P, I64, P, P, P, I64, I64, I32, I32, I32, F32, P]),
    "aacc_rmsnorm": (I32, [P, P, P, I64, I64, F32, P]),
    "aacc_add_rmsnorm": (I32, [P, P, P, P, I64, I64, F32, P]),
    "aacc_embed_rmsnorm": (I32, [P, P, I64, P, P, P, I64, I64, F32, P]),
    "aacc_gemm": (I32, [P, P, P, I64, I64, I64, P]),
    "aacc_gemm_silu_mul": (I32, [P, P, P, I64, I64, I64, P]),
    "aacc_gemm_splitk": (I32, [P, P, P, I64, I64, I64, I32, P]),
    "aacc_gemm_bias": (I32, [P, P, P, P, I64, I64, I64, P]),
    "aacc_gemm_cluster": (I32, [P, P, P, I64, I64, I64, I32, P]),
    "aacc_gemm_silu_mul_cluster": (I32, [P, P, P, I64, I64, I64, I32, P]),
    "aacc_qkv_norm_rope_store_cluster": (I32, [P, P, P, P, F32, P, P, I64, P, P, P, P, I64, I32, I32, I32, I64, I64,
                                               I32, P]),
    "aacc_gemm_cluster_plan": (I32, [I64, I64, I64, P, P, P]),
    "aacc_gemm_cluster_capacity": (I64, [I32, I32]),
    "aacc_gemm_skinny_splitk": (I32, [P, P, P, I64, I64, I64, I32, P]),
    "aacc_skinny_qkv_norm_rope_store": (I32, [P, P, P, I32, P, P, P, F32, P, P, I64, P, P, P, P, I64, I32, I32, I32,
                                              I64, I64, P]),
    "aacc_skinny_silu_mul": (I32, [P, P, P, I32, P, P, I64, I64, I64, P]),
    "aacc_bias_add": (I32, [P, P, I64, I64, P]),
    "aacc_splitk_add_rmsnorm": (I32, [P, I32, P, P, P, I64, I64, F32, P]),
    "aacc_splitk_reduce": (I32, [P, I32, P, I64, I64, P]),
    "aacc_splitk_qkv_norm_rope_store": (I32, [P, I32, P, P, F32, P, P, I64, P, P, P, P, I64, I32, I32, I32, I64,
                                              P]),
    "aacc_splitk_silu_mul": (I32, [P, I32, P, I64, I64, P]),
    "aacc_qkv_norm_rope_store": (I32, [P, P, P, P, F32, P, P, I64, P, P, P, P, I64, I32, I32, I32, I64, I64, P]),
    "aacc_lm_head_workspace_bytes": (I64, [I64, I64]),
    "aacc_lm_head_argmax": (I32, [P, P, I64, I64, I64, I64, P, P, P, P, I64, P]),
    "aacc_lm_head_sample": (I32, [P, P, I64, I64, I64, I64, P, P, P, P, P, P, P, I64, P]),
    "aacc_argmax_rows": (I32, [P, I64, I64, P, P]),
    "aacc_sample_rows": (I32, [P, I64, I64, P, P, P, P, P]),
    "aacc_argmax_merge": (I32, [P, P, I64, I32, P, P]),
    "aacc_argmax_merge_strided": (I32, [P, P, I64, I32, I64, I64, P, P]),
    "aacc_tp_set_peer_wait_ms": (I32, [I64]),
    "aacc_tp_exchange_bytes": (I64, [I32, I64, I64]),
    "aacc_peer_buffer_alloc": (I32, [I64, P, P]),
    "aacc_peer_buffer_open": (I32, [P, P]),
    "aacc_peer_buffer_close": (I32, [P]),
    "aacc_peer_buffer_free": (I32, [P]),
    "aacc_tp_allreduce_add_rmsnorm": (I32, [P, I32, P, I32, I32, I32, I64, P, P, P, I64, I64, F32, P]),
}

_lib = None


def load() -> ctypes.CDLL:
    """Load (once) and return the kernel library; raise if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"B200 kernel library not built ({LIB_PATH}); run `python -m awesome_acceleration_b200.build`")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int, what: str) -> None:
    if status != 0:
        msg = load().aacc_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed (status {status}): {msg}")


def device_error() -> int:
    """Read the device error word (bound violations / wait timeouts), synchronising."""
    v = ctypes.c_uint(0)
    check(load().aacc_get_device_error(ctypes.byref(v)), "aacc_get_device_error")
    return int(v.value)


def clear_device_error() -> None:
    check(load().aacc_clear_device_error(), "aacc_clear_device_error")


DEVICE_ERRORS = {1: "block id outside the KV pool", 2: "cache slot outside the KV pool",
                 4: "device wait timed out", 8: "position outside the RoPE table",
                 16: "token id outside the vocabulary", 32: "context longer than the block table",
                 64: "a peer GPU did not arrive in the TP exchange"}


def raise_on_device_error(what: str = "kernel") -> None:
    e = device_error()
    if e:
        reasons = ", ".join(v for k, v in DEVICE_ERRORS.items() if e & k)
        clear_device_error()
        raise RuntimeError(f"{what}: device error 0x{e:x} ({reasons})")
