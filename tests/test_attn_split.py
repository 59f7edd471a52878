"""The split decode attention's arithmetic on the CPU (numpy), as k_sdpa_part /
k_sdpa_merge do it: the positions 0..n-1 of a token are cut into S splits of
ceil(n / S) positions, the splits that hold positions are exactly the first
ceil(n / chunk), they cover every position once; and the per-split online
softmax (128-position passes, running maximum and sum, rescaled accumulator)
merged at the common maximum equals the single-pass softmax-weighted sum."""
import numpy as np
import pytest


def splits(n, S):
    chunk = (n + S - 1) // S
    ranges = [(s * chunk, min(n, s * chunk + chunk)) for s in range(S)]
    used = (n + chunk - 1) // chunk
    return chunk, used, ranges


def test_partition_covers_every_position_once():
    for S in range(1, 33):
        for n in range(1, 700):
            chunk, used, ranges = splits(n, S)
            held = [s for s, (a, b) in enumerate(ranges) if a < b]
            assert held == list(range(used)), (n, S)
            covered = np.concatenate([np.arange(a, b) for a, b in ranges if a < b])
            assert np.array_equal(covered, np.arange(n)), (n, S)


def part(scores, v, a, b, tile=128):
    """One split: online softmax over [a, b) in passes of `tile` positions (float32)."""
    m, l = np.float32(-np.inf), np.float32(0)
    acc = np.zeros(v.shape[1], np.float32)
    for j0 in range(a, b, tile):
        s = scores[j0:min(b, j0 + tile)]
        m_new = np.float32(max(m, s.max()))
        p = np.exp(s - m_new).astype(np.float32)
        corr = np.float32(np.exp(m - m_new))
        l = np.float32(l * corr + p.sum(dtype=np.float32))
        acc = (acc * corr + p @ v[j0:j0 + len(s)]).astype(np.float32)
        m = m_new
    return m, l, acc


@pytest.mark.parametrize("n,S", [(1, 32), (7, 32), (65, 32), (2049, 32), (2049, 10), (3000, 1), (129, 2)])
def test_split_merge_equals_single_pass(n, S):
    rng = np.random.default_rng(n * 31 + S)
    scores = (rng.standard_normal(n) * 4).astype(np.float32)
    v = rng.standard_normal((n, 128)).astype(np.float32)
    _, used, ranges = splits(n, S)
    parts = [part(scores, v, a, b) for a, b in ranges[:used]]
    M = max(p[0] for p in parts)
    w = [np.float32(np.exp(p[0] - M)) for p in parts]
    L = sum(wi * p[1] for wi, p in zip(w, parts))
    out = sum(wi * p[2] for wi, p in zip(w, parts)) / L
    e = np.exp(scores.astype(np.float64) - scores.max())
    ref = (e / e.sum()) @ v.astype(np.float64)
    assert np.max(np.abs(out - ref)) <= 1e-5 * max(1.0, np.max(np.abs(ref)))
