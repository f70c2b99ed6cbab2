"""Cross-process KV hand-off over CUDA IPC (a prefill engine's request KV into
a decode engine's paged cache).

The reference disaggregates prefill and decode by exporting a request's
per-layer K/V to host tensors (``export_request_kv``, model/model.py:156-166,
:386-390) and shipping them through host shared memory between processes
(pd/kv_connector_shm.py:97-209, llm_pd.py:195-340); the decode side copies
them back into its cache (``import_request_kv``, model/model.py:168-177,
:392-401).  Here the K/V never touch host memory:

  prefill process   ``export_request_kv_ipc`` gathers the request's K/V of
                    every layer into ONE device buffer made with
                    ``aacc_peer_buffer_alloc`` (a dedicated cudaMalloc whose
                    CUDA IPC handle maps exactly that buffer) and returns a
                    small picklable ``KVTicket`` (the 64-byte handle + sizes)
                    and an ``ExportedKV`` that owns the buffer;
  decode process    ``import_request_kv_ipc`` opens the buffer
                    (``aacc_peer_buffer_open``: the same GPU, or another GPU
                    of the node, read over NVLink), stores it into its own
                    paged cache with the ``kv_store`` kernel reading the
                    mapped memory directly, waits for the copy, and closes
                    the mapping;
  prefill process   ``ExportedKV.release()`` frees the buffer once the decode
                    side has acknowledged (through whatever channel carried
                    the ticket).

Buffer layout: bf16 ``[2][layers][length][kv_heads][128]`` (K, then V).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from . import kernels as K


@dataclass(frozen=True)
class KVTicket:
    """What the decode side needs to open and import an exported request."""
    handle: bytes      # 64-byte CUDA IPC memory handle
    nbytes: int
    layers: int
    length: int        # tokens exported
    kv_heads: int
    seqlen: int        # the sequence's length in the exporting cache


class _DeviceView:
    """Zero-copy torch view of a device buffer this process owns (CUDA array interface)."""

    def __init__(self, ptr: int, nelem: int):
        self.__cuda_array_interface__ = {"shape": (nelem,), "typestr": "<i2", "data": (ptr, False), "version": 3,
                                         "strides": None}


def _as_bf16(ptr: int, shape: tuple[int, ...], device) -> torch.Tensor:
    n = int(np.prod(shape))
    return torch.as_tensor(_DeviceView(ptr, n), device=device).view(torch.bfloat16).view(shape)


class ExportedKV:
    """Owns the exported buffer until ``release()`` (after the importer is done)."""

    def __init__(self, ptr: int, device: torch.device):
        self.ptr, self.device = ptr, device

    def release(self) -> None:
        if self.ptr is not None:
            with torch.cuda.device(self.device):
                torch.cuda.synchronize()
                K.peer_buffer_free(self.ptr)
            self.ptr = None


def export_request_kv_ipc(model, slot_idx: int, length: int) -> tuple[KVTicket, ExportedKV]:
    """Gather the first ``length`` tokens of ``slot_idx`` (every layer) into an
    IPC-exportable device buffer; returns the ticket to send and the owner."""
    kv = model.kv
    L, hkv, length = kv.num_layers, kv.num_kv_heads, int(length)
    if length <= 0 or length > int(kv.lengths[int(slot_idx)]):
        raise ValueError(f"export_request_kv_ipc: length {length} outside the slot's {int(kv.lengths[int(slot_idx)])}"
                         f" cached tokens")
    dev = kv.k.device
    shape = (2, L, length, hkv, 128)
    nbytes = int(np.prod(shape)) * 2
    with torch.cuda.device(dev):
        ptr, handle = K.peer_buffer_alloc(nbytes)
        try:
            buf = _as_bf16(ptr, shape, dev)
            for i in range(L):
                k, v = kv.gather(i, int(slot_idx), length)
                buf[0, i].copy_(k)
                buf[1, i].copy_(v)
            torch.cuda.current_stream().synchronize()  # the importer reads it from another process
        except BaseException:
            K.peer_buffer_free(ptr)
            raise
    ticket = KVTicket(handle=handle, nbytes=nbytes, layers=L, length=length, kv_heads=hkv,
                      seqlen=int(kv.lengths[int(slot_idx)]))
    return ticket, ExportedKV(ptr, dev)


def import_request_kv_ipc(model, slot_idx: int, ticket: KVTicket) -> None:
    """Open an exported buffer and store it into ``slot_idx`` of this model's
    paged cache (the ``import_request_kv`` contract: the slot's length becomes
    the exporter's sequence length)."""
    kv = model.kv
    if ticket.layers != kv.num_layers or ticket.kv_heads != kv.num_kv_heads:
        raise ValueError(f"import_request_kv_ipc: payload has {ticket.layers} layers x {ticket.kv_heads} kv heads, "
                         f"the cache {kv.num_layers} x {kv.num_kv_heads}")
    row, n = int(slot_idx), ticket.length
    dev = kv.k.device
    with torch.cuda.device(dev):
        kv.reserve(row, n)
        kv.sync()
        slots = torch.from_numpy(kv.slot_mapping(row, 0, n)).to(dev)
        ptr = K.peer_buffer_open(ticket.handle)
        try:
            lib = _lib.load()
            stream = torch.cuda.current_stream().cuda_stream
            layer_bytes = n * kv.num_kv_heads * 128 * 2
            rs = kv.num_kv_heads * 128  # row stride of one token, elements
            nb, hkv, bs, _ = kv.k[0].shape
            for i in range(kv.num_layers):
                k_ptr = ptr + i * layer_bytes
                v_ptr = ptr + (kv.num_layers + i) * layer_bytes
                _lib.check(lib.aacc_kv_store(k_ptr, v_ptr, n, rs, rs, slots.data_ptr(), kv.k[i].data_ptr(),
                                             kv.v[i].data_ptr(), nb, hkv, bs, stream), "kv_store (ipc import)")
            torch.cuda.current_stream().synchronize()  # done reading the peer buffer
        finally:
            K.peer_buffer_close(ptr)
        kv.set_lengths([row], [ticket.seqlen])
