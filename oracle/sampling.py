"""CPU restatement of temperature sampling (test infrastructure).

The reference samples ``torch.multinomial(F.softmax(logits / T, dim=-1), 1)``
(llm.py:215-219, llm_tp.py:609-616); ``logits / T`` is a bf16 tensor op, so
the distribution it draws from is softmax(bf16(logits / T)).
``reference_probs`` gives that distribution.

The B200 kernels draw from the same distribution with the Gumbel-max trick:
token = argmax_v bf16(logit_v / T) + G_v with counter-based standard Gumbel
noise G.  ``gumbel_noise`` / ``sample`` restate that draw bit for bit in
numpy (SplitMix64 output function of Steele, Lea and Flood, OOPSLA 2014;
32-bit finaliser of Appleby's MurmurHash3), so tests can check the kernel's
tokens row by row as well as their distribution.
"""
from __future__ import annotations

import numpy as np
import torch


def _splitmix64(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = x.astype(np.uint64) + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def _fmix32(h: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        h = h.astype(np.uint32)
        h ^= h >> np.uint32(16)
        h *= np.uint32(0x85EBCA6B)
        h ^= h >> np.uint32(13)
        h *= np.uint32(0xC2B2AE35)
        h ^= h >> np.uint32(16)
        return h


def sample_key(seeds, counters) -> np.ndarray:
    """Per-row noise key: splitmix64(seed ^ splitmix64(counter))."""
    s = np.asarray(seeds, dtype=np.int64).view(np.uint64)
    c = np.asarray(counters, dtype=np.int64).view(np.uint64)
    return _splitmix64(s ^ _splitmix64(c))


def gumbel_noise(key: np.ndarray, vocab_ids: np.ndarray) -> np.ndarray:
    """[rows, len(vocab_ids)] fp32 standard Gumbel noise."""
    key = np.asarray(key, dtype=np.uint64)[:, None]
    v = np.asarray(vocab_ids, dtype=np.uint32)[None, :]
    with np.errstate(over="ignore"):
        lo = (key & np.uint64(0xFFFFFFFF)).astype(np.uint32)
        hi = (key >> np.uint64(32)).astype(np.uint32)
        h = _fmix32(_fmix32(lo ^ (v * np.uint32(0x9E3779B9))) + hi)
    u = ((h >> np.uint32(8)).astype(np.float32) + np.float32(0.5)) * np.float32(1.0 / 16777216.0)
    return (-np.log(-np.log(u))).astype(np.float32)


def _bf16(x: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).bfloat16().float().numpy()


def sample(logits, temperatures, seeds, counters, vocab_offset: int = 0) -> np.ndarray:
    """The kernels' draw over bf16 logits [rows, V]: argmax of bf16(logit / T)
    + noise (lowest id on ties); rows with T <= 0 take the plain argmax.
    Returns global ids (column + vocab_offset)."""
    lg = _bf16(np.asarray(logits, dtype=np.float32))
    t = np.asarray(temperatures, dtype=np.float32)
    out = lg.argmax(axis=1).astype(np.int64)
    hot = t > 0
    if hot.any():
        ids = np.arange(lg.shape[1]) + vocab_offset
        noise = gumbel_noise(sample_key(np.asarray(seeds)[hot], np.asarray(counters)[hot]), ids)
        score = _bf16(lg[hot] / t[hot, None]) + noise
        out[hot] = score.argmax(axis=1)
    return out + vocab_offset


def reference_probs(logits_row, temperature: float) -> np.ndarray:
    """softmax(bf16(logits / T)) in fp64: the distribution the reference draws from."""
    z = _bf16(np.asarray(logits_row, dtype=np.float32) / np.float32(temperature)).astype(np.float64)
    z -= z.max()
    p = np.exp(z)
    return p / p.sum()
