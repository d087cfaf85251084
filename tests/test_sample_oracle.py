"""The sampler's CPU restatement (``oracle/sample.py``) against a literal
numpy transcription of the reference's sampled branch
(worker/executor.py:270-306: descending argsort, cumsum, ``cumsum <= top_p``
shifted right with the first token kept, renormalise), on CPU."""

import numpy as np
import pytest

from oracle import sample as osample


def reference_kept(logits, T, top_p):
    """executor.py:280-297 step by step (float64): the renormalised masked
    distribution scattered back to vocabulary order."""
    z = logits / T
    probs = np.exp(z - z.max(axis=-1, keepdims=True))
    probs /= probs.sum(axis=-1, keepdims=True)
    idx = np.argsort(probs, axis=-1)[:, ::-1]
    sp = np.take_along_axis(probs, idx, axis=-1)
    mask = np.cumsum(sp, axis=-1) <= top_p
    mask = np.concatenate([np.ones((mask.shape[0], 1), bool), mask[:, :-1]], axis=-1)
    mp = np.where(mask, sp, 0.0)
    mp /= mp.sum(axis=-1, keepdims=True)
    out = np.zeros_like(probs)
    np.put_along_axis(out, idx, mp, axis=-1)
    return out


@pytest.mark.parametrize("V", [7, 1000, 32000])
@pytest.mark.parametrize("T,p", [(0.7, 0.9), (1.0, 0.5), (1.5, 1.0), (0.3, 0.95), (1.0, 1e-6)])
def test_kept_distribution_matches_the_reference_steps(V, T, p):
    rng = np.random.default_rng(V)
    logits = rng.standard_normal((8, V)) * 3
    ref = reference_kept(logits, T, p)
    got = osample.kept_distribution(logits, T, p)
    np.testing.assert_allclose(got, ref, rtol=1e-12, atol=1e-15)


def test_draw_is_the_inverse_cdf_of_the_kept_distribution():
    rng = np.random.default_rng(5)
    V, T, p = 50, 0.8, 0.9
    row = rng.standard_normal(V) * 2
    q = osample.kept_distribution(row[None], T, p)[0]
    u = (np.arange(4000) + 0.5) / 4000
    toks = osample.draw(np.tile(row, (u.size, 1)), T, p, u)
    freq = np.bincount(toks, minlength=V) / u.size
    assert np.max(np.abs(freq - q)) <= 1.0 / u.size + 1e-12
    assert np.all(freq[q == 0] == 0)


def test_top_p_keeps_at_least_the_most_likely_token():
    logits = np.array([[0.0, 5.0, 1.0, 4.9]])
    k = osample.kept_mask(osample.softmax_t(logits, 1.0), 1e-9)
    assert k.tolist() == [[False, True, False, False]]
    assert osample.draw(logits, 1.0, 1e-9, [0.999])[0] == 1
