"""TP / DP x TP process groups and collectives (the reference's L0 runtime).

Mirrors yijichar/AWesome_ACceleration model/distributed.py: the same
``init_distributed(tp_size, backend)`` layout (world split into TP groups of
consecutive ranks with an NCCL group for tensors and a Gloo group for
pickled control messages, plus strided DP groups, :39-95), the same query
functions (:100-141) and collective helpers (:151-235).

Differences: ``init_distributed`` takes a ``timeout`` (so a rank that died
turns the others' next collective into an error instead of a hang) and works
with ``backend="gloo"`` on CPU-only hosts (used by the multi-rank tests);
``tensor_model_parallel_all_gather`` gathers into one preallocated tensor.
"""
from __future__ import annotations

import datetime
import os
from typing import Optional

import torch
import torch.distributed as dist

_GLOBAL_TP_PROFILER = None

_TP_GROUP: Optional[dist.ProcessGroup] = None
_DP_GROUP: Optional[dist.ProcessGroup] = None
_TP_CPU_GROUP: Optional[dist.ProcessGroup] = None
_WORLD_SIZE = 1
_GLOBAL_RANK = 0
_LOCAL_RANK = 0
_TP_WORLD_SIZE = 1
_TP_RANK = 0
_DP_WORLD_SIZE = 1
_DP_RANK = 0
_TP_LEADER_GLOBAL_RANK = 0


def set_tp_profiler(profiler):
    global _GLOBAL_TP_PROFILER
    _GLOBAL_TP_PROFILER = profiler


def init_distributed(tp_size: int, backend: str = "nccl", timeout_s: float = 300.0):
    """World -> TP groups of consecutive ranks (+ Gloo twins) and strided DP groups
    (model/distributed.py:39-95)."""
    global _TP_GROUP, _DP_GROUP, _TP_CPU_GROUP, _WORLD_SIZE, _GLOBAL_RANK, _LOCAL_RANK
    global _TP_WORLD_SIZE, _TP_RANK, _DP_WORLD_SIZE, _DP_RANK, _TP_LEADER_GLOBAL_RANK
    timeout = datetime.timedelta(seconds=timeout_s)
    _LOCAL_RANK = int(os.environ.get("LOCAL_RANK", 0))
    if not dist.is_initialized():
        kw = {}
        if backend == "nccl":
            torch.cuda.set_device(_LOCAL_RANK)
            kw["device_id"] = torch.device("cuda", _LOCAL_RANK)
        dist.init_process_group(backend=backend, timeout=timeout, **kw)
    _WORLD_SIZE = dist.get_world_size()
    _GLOBAL_RANK = dist.get_rank()
    if _WORLD_SIZE % tp_size:
        raise ValueError(f"WORLD_SIZE ({_WORLD_SIZE}) must be divisible by tp_size ({tp_size})")
    _TP_WORLD_SIZE = tp_size
    _DP_WORLD_SIZE = _WORLD_SIZE // tp_size
    _TP_RANK = _GLOBAL_RANK % tp_size
    _DP_RANK = _GLOBAL_RANK // tp_size
    if backend == "nccl":
        torch.cuda.set_device(_LOCAL_RANK)
    tp_lists = [list(range(r * tp_size, (r + 1) * tp_size)) for r in range(_DP_WORLD_SIZE)]
    for ranks in tp_lists:  # every rank creates every group, in the same order
        g = dist.new_group(ranks=ranks, backend=backend, timeout=timeout)
        if _GLOBAL_RANK in ranks:
            _TP_GROUP, _TP_LEADER_GLOBAL_RANK = g, ranks[0]
    for ranks in tp_lists:
        g = dist.new_group(ranks=ranks, backend="gloo", timeout=timeout)
        if _GLOBAL_RANK in ranks:
            _TP_CPU_GROUP = g
    for t in range(tp_size):
        ranks = [r * tp_size + t for r in range(_DP_WORLD_SIZE)]
        g = dist.new_group(ranks=ranks, backend=backend, timeout=timeout)
        if _GLOBAL_RANK in ranks:
            _DP_GROUP = g


def reset_distributed_state():
    """Forget the groups (tests that re-initialise in one process)."""
    global _TP_GROUP, _DP_GROUP, _TP_CPU_GROUP, _WORLD_SIZE, _GLOBAL_RANK, _TP_WORLD_SIZE, _TP_RANK
    global _DP_WORLD_SIZE, _DP_RANK, _TP_LEADER_GLOBAL_RANK
    _TP_GROUP = _DP_GROUP = _TP_CPU_GROUP = None
    _WORLD_SIZE = _TP_WORLD_SIZE = _DP_WORLD_SIZE = 1
    _GLOBAL_RANK = _TP_RANK = _DP_RANK = _TP_LEADER_GLOBAL_RANK = 0


# ------------------------------------------------------------------ queries (:100-141)
def get_world_size() -> int:
    return _WORLD_SIZE


def get_global_rank() -> int:
    return _GLOBAL_RANK


def get_dp_world_size() -> int:
    return _DP_WORLD_SIZE


def get_dp_rank() -> int:
    return _DP_RANK


def get_dp_group():
    return _DP_GROUP


def is_tp_leader() -> bool:
    return _TP_RANK == 0


def get_tp_leader_global_rank() -> int:
    return _TP_LEADER_GLOBAL_RANK


def is_global_rank_0() -> bool:
    return _GLOBAL_RANK == 0


def is_distributed() -> bool:
    """True when TP collectives are needed (tp_size > 1), as in the reference."""
    return _TP_WORLD_SIZE > 1


def get_tp_world_size() -> int:
    return _TP_WORLD_SIZE


def get_tp_rank() -> int:
    return _TP_RANK


def get_local_rank() -> int:
    return _LOCAL_RANK


def is_tp_rank_0() -> bool:
    return _TP_RANK == 0


def get_tp_group():
    return _TP_GROUP


def get_tp_cpu_group():
    return _TP_CPU_GROUP


# ------------------------------------------------------------------ collectives (:151-217)
def _section(name):
    prof = _GLOBAL_TP_PROFILER
    if prof is not None and getattr(prof, "enabled", False):
        return prof.section(name)
    return None


def tensor_model_parallel_all_reduce(input_: torch.Tensor) -> torch.Tensor:
    if not is_distributed():
        return input_
    sec = _section("comm.all_reduce")
    if sec is None:
        dist.all_reduce(input_, group=_TP_GROUP)
    else:
        with sec:
            dist.all_reduce(input_, group=_TP_GROUP)
    return input_


def tensor_model_parallel_all_gather(input_: torch.Tensor, dim: int = -1) -> torch.Tensor:
    if not is_distributed():
        return input_
    t = _TP_WORLD_SIZE
    out = torch.empty((t,) + tuple(input_.shape), dtype=input_.dtype, device=input_.device)
    dist.all_gather_into_tensor(out, input_.contiguous(), group=_TP_GROUP)
    dim = dim % input_.dim()
    return torch.cat(list(out.unbind(0)), dim=dim)


def broadcast_tensor(tensor: torch.Tensor, src: int = 0) -> torch.Tensor:
    if not is_distributed():
        return tensor
    dist.broadcast(tensor, src=_TP_LEADER_GLOBAL_RANK + src, group=_TP_GROUP)
    return tensor


def broadcast_object(obj, src: int = 0):
    """Pickled control message over the TP Gloo group (model/distributed.py:199-217)."""
    if not is_distributed():
        return obj
    if _TP_CPU_GROUP is None:
        raise RuntimeError("TP CPU control group is not initialized")
    lst = [obj]
    dist.broadcast_object_list(lst, src=_TP_LEADER_GLOBAL_RANK + src, group=_TP_CPU_GROUP)
    return lst[0]


def split_tensor_along_dim(tensor: torch.Tensor, num_partitions: int, dim: int,
                           contiguous: bool = True) -> torch.Tensor:
    """This rank's chunk (model/distributed.py:222-235)."""
    if tensor.shape[dim] % num_partitions:
        raise ValueError(f"Dimension {dim} ({tensor.shape[dim]}) not divisible by {num_partitions}")
    out = torch.chunk(tensor, num_partitions, dim=dim)[get_tp_rank()]
    return out.contiguous() if contiguous else out


def gather_from_tensor_model_parallel_region(input_: torch.Tensor, dim: int = -1) -> torch.Tensor:
    return tensor_model_parallel_all_gather(input_, dim=dim)


class SyncMode:
    """TP barrier context (model/distributed.py:245-254)."""

    def __enter__(self):
        if is_distributed():
            dist.barrier(group=_TP_GROUP)
        return self

    def __exit__(self, *a):
        if is_distributed():
            dist.barrier(group=_TP_GROUP)
        return False
