"""B200-native (sm_100a) per-step hot path of the Qwen3 inference engine of
yijichar/AWesome_ACceleration, behind the reference's Python API.

    from awesome_acceleration_b200 import LLM            # llm.py
    from awesome_acceleration_b200.llm_tp import LLMTP   # llm_tp.py
    from awesome_acceleration_b200.model.model import Qwen3ForCausalLM, Qwen3Config
    from awesome_acceleration_b200.model.parallel_layers import (
        ColumnParallelLinear, RowParallelLinear, QKVParallelLinear)

The kernels live in ``libaacc_b200.so`` (C ABI: ``include/aacc_b200.h``),
built in-tree by ``python -m awesome_acceleration_b200.build``.
"""
from __future__ import annotations

__all__ = ["LLM", "GenerationOutput", "Qwen3Config", "Qwen3ForCausalLM"]


def __getattr__(name):
    if name in ("LLM", "GenerationOutput"):
        from . import llm
        return getattr(llm, name)
    if name in ("Qwen3Config", "Qwen3ForCausalLM"):
        from .model import model
        return getattr(model, name)
    raise AttributeError(name)
