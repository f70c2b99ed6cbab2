import json
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built kernel library")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def load_golden(name: str) -> dict:
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"), allow_pickle=False)
    d = {k: z[k] for k in z.files}
    d["arch"] = json.loads(str(d["arch"]))
    d["dtype"] = str(d["dtype"])
    return d


def load_gpuref(name: str) -> dict | None:
    """The reference path run with cuBLAS on a B200 for golden `name`
    (tests/golden/make_gpu_reference.py), or None if it was not recorded."""
    path = os.path.join(GOLDEN, f"{name}_gpuref.npz")
    if not os.path.exists(path):
        return None
    z = np.load(path, allow_pickle=False)
    return {k: z[k] for k in z.files}


def bf16_ulp(x: np.ndarray) -> np.ndarray:
    """Spacing of bf16 values at |x| (8 significant bits)."""
    ax = np.maximum(np.abs(x.astype(np.float64)), 2.0 ** -126)
    return 2.0 ** (np.floor(np.log2(ax)) - 7)


def build_model(arch, sd: dict, num_slots: int, max_seq_len: int, dev, **kw):
    """Single-GPU B200 model with the seeded weights `sd` (bf16), fused, KV cache allocated."""
    import torch
    from awesome_acceleration_b200.model.model import Qwen3Config, Qwen3ForCausalLM
    cfg = Qwen3Config(**{k: v for k, v in arch.as_dict().items() if k in Qwen3Config.__annotations__})
    with torch.device("meta"):
        m = Qwen3ForCausalLM(cfg)
    m = m.to_empty(device=dev).to(torch.bfloat16)
    missing, unexpected = m.load_state_dict({k: v.to(torch.bfloat16) for k, v in sd.items()}, strict=False)
    assert not unexpected
    block_size = kw.pop("block_size", 256)
    for k, v in kw.items():
        setattr(m, k, v)
    m.fuse_qkv()
    m.init_kv_cache(num_slots, max_seq_len, dev, torch.bfloat16, block_size=block_size)
    return m


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from awesome_acceleration_b200 import _lib
    _lib.load()
    return torch.device("cuda")
