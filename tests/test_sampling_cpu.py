"""The sampling pipeline's host pieces, on CPU: DeterministicRng (product host
logic) against the oracle's restatement, the SplitMix64 seeding pinned to its
published first output, and the oracle sampler's defining properties
(InferenceSession.cs:565-734)."""
import numpy as np
import pytest


def test_splitmix64_published_first_output():
    # SplitMix64 from state 0 returns 0xE220A8397B1DCDAF first (the generator's published reference output)
    M = (1 << 64) - 1
    s = 0x9E3779B97F4A7C15
    z = ((s ^ (s >> 30)) * 0xBF58476D1CE4E5B9) & M
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
    assert z ^ (z >> 31) == 0xE220A8397B1DCDAF


@pytest.mark.parametrize("seed", [0, 1, 42, -7, 2**31 - 1])
def test_deterministic_rng_matches_oracle(O, seed):
    from smallmind_b200.api import DeterministicRng
    r = DeterministicRng(seed)
    got = np.array([r.next_double() for _ in range(64)])
    assert np.array_equal(got, O.deterministic_rng_doubles(seed, 64))
    assert np.all((got >= 0) & (got < 1))


def test_oracle_sampler_properties(O):
    rs = np.random.RandomState(0)
    lg = rs.randn(500).astype(np.float32)
    am = int(np.argmax(lg))
    for tgt in (1e-9, 0.3, 0.999999):  # (a target of exactly 0 picks index 0, as in the reference)
        assert O.sample(lg, tgt, top_k=1)[0] == am  # TopK = 1 is greedy
        assert O.sample(lg, tgt, top_p=1e-6)[0] == am
    t, p = O.sample(lg, 0.5)
    assert abs(float(p.sum()) - 1.0) < 1e-5 and p.min() > 0
    # top-k keeps exactly k nonzero probabilities (no ties in randn)
    _, p = O.sample(lg, 0.5, top_k=17)
    assert np.count_nonzero(p) == 17 and set(np.nonzero(p)[0]) == set(np.argsort(-lg)[:17])
    # min-p drops everything under min_p * max
    _, p = O.sample(lg, 0.5, min_p=0.2)
    kept = p > 0
    base = np.exp(lg - lg.max())
    assert np.array_equal(kept, base >= 0.2 * base.max() * (1 - 1e-6)) or abs(int(kept.sum()) - int((base >= 0.2 * base.max()).sum())) <= 1
    # repetition penalty divides positive and multiplies negative logits of seen tokens (:829-839)
    x = np.array([2.0, -2.0, 1.0, 0.5], np.float32)
    _, p = O.sample(x.copy(), 0.5, repetition_penalty=2.0, context=[0, 1, 1])
    y = np.array([1.0, -4.0, 1.0, 0.5], np.float32)
    e = np.exp(y - y.max())
    assert np.allclose(p, e / e.sum(), rtol=1e-6)
    # frequency penalty subtracts count * penalty, presence penalty once per distinct token
    _, p = O.sample(x.copy(), 0.5, presence_penalty=0.5, frequency_penalty=0.25, context=[2, 2, 2, 3])
    y = np.array([2.0, -2.0, 1.0 - 0.5 - 0.75, 0.5 - 0.5 - 0.25], np.float32)
    e = np.exp(y - y.max())
    assert np.allclose(p, e / e.sum(), rtol=1e-6)
    # the target picks the first index whose cumulative sum reaches it (:714-734)
    _, p = O.sample(lg, 0.0)
    c = np.cumsum(p.astype(np.float64))
    for tgt in (0.1, 0.5, 0.9):
        assert O.sample(lg, tgt)[0] == int(np.argmax(c >= tgt))
