"""The sampling oracle: Philox4x32-10 against the generator's published
known-answer vectors, and the Gumbel-max sampler against the distribution it
must draw from (softmax(logits / T), the reference's sample() without top_k,
generate.py:46-63)."""
import numpy as np

from oracle.sample_oracle import gumbel_noise, philox4x32_10, sample_token

# Known-answer vectors of Philox4x32-10 (Random123 distribution, kat_vectors).
KAT = [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF), (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


def test_philox_known_answers():
    for ctr, key, want in KAT:
        assert philox4x32_10(ctr, key) == want


def test_vectorised_noise_matches_scalar_generator():
    rows = np.array([0, 1, 7, 123456, 2 ** 31 - 1], dtype=np.int64)
    g = gumbel_noise(rows, pos=513, seed=0x1234_5678_9ABC_DEF0)
    for r, v in zip(rows, g):
        w = philox4x32_10((int(r), 513, 0, 0x5EED5A3B), (0x9ABCDEF0, 0x12345678))[0]
        u = ((w >> 8) + 0.5) / 16777216.0
        assert abs(v - (-np.log(-np.log(u)))) < 1e-5


def test_gumbel_max_draws_softmax():
    """Frequencies over 20000 positions match softmax(logits / T) (chi-square)."""
    logits = np.array([1.0, 0.5, 0.0, -0.5, 2.0, 1.5, -1.0, 0.25], dtype=np.float16)
    T = 0.8
    n = 20000
    counts = np.zeros(len(logits))
    for pos in range(n):
        counts[sample_token(logits, T, pos, seed=99)] += 1
    p = np.exp(logits.astype(np.float64) / T)
    p /= p.sum()
    chi2 = float(((counts - n * p) ** 2 / (n * p)).sum())
    assert chi2 < 30.0, (chi2, counts / n, p)  # 7 degrees of freedom: p-value ~ 1e-4
