"""Temperature sampling oracle on the CPU: the counter-based Gumbel-max draw
the kernels implement samples the reference's distribution
softmax(bf16(logits / T)) (llm.py:215-219)."""
import numpy as np

from oracle.sampling import gumbel_noise, reference_probs, sample, sample_key


def test_gumbel_noise_moments():
    key = sample_key(np.arange(64), np.full(64, 7))
    g = gumbel_noise(key, np.arange(4096)).astype(np.float64).ravel()
    assert abs(g.mean() - 0.5772156649) < 0.01          # Euler-Mascheroni constant
    assert abs(g.var() - np.pi ** 2 / 6) < 0.03
    # streams for different counters / seeds are not the same numbers
    assert not np.array_equal(gumbel_noise(sample_key([1], [0]), np.arange(64)),
                              gumbel_noise(sample_key([1], [1]), np.arange(64)))


def test_gumbel_max_matches_reference_distribution():
    rng = np.random.default_rng(3)
    V, rows, T = 48, 40000, 0.7
    logits = (rng.standard_normal(V) * 2).astype(np.float32)
    toks = sample(np.tile(logits, (rows, 1)), np.full(rows, T), np.arange(rows), np.full(rows, 5))
    emp = np.bincount(toks, minlength=V) / rows
    p = reference_probs(logits, T)
    tv = 0.5 * np.abs(emp - p).sum()
    assert tv < 0.02, tv
    keep = p * rows >= 20
    chi2 = ((emp[keep] * rows - p[keep] * rows) ** 2 / (p[keep] * rows)).sum()
    assert chi2 < 3 * keep.sum(), (chi2, keep.sum())


def test_greedy_rows_and_vocab_shards():
    rng = np.random.default_rng(4)
    lg = rng.standard_normal((16, 256)).astype(np.float32)
    t = np.where(np.arange(16) % 2 == 0, 0.0, 1.3)
    full = sample(lg, t, np.arange(16), np.arange(16))
    assert np.array_equal(full[::2], lg[::2].argmax(1))  # T = 0 rows are greedy
    # two vocab shards, each perturbed with its global ids: one of them holds the draw
    a = sample(lg[:, :128], t, np.arange(16), np.arange(16), vocab_offset=0)
    b = sample(lg[:, 128:], t, np.arange(16), np.arange(16), vocab_offset=128)
    assert np.all((full == a) | (full == b))
