"""Temperature + top-p sampling of the reference, restated in numpy (float64).

TEST INFRASTRUCTURE ONLY (used by ``tests/``), never by the product package.

Reference: ``worker/executor.py:270-306`` (the sampled branch of
``ParallelExecutor.generate``):

* ``logits / temperature``; ``probs = softmax``;
* sort descending; ``cumsum``; token ``i`` of the sorted order is kept when
  the mass of the tokens sorted before it is ``<= top_p`` (the reference's
  ``mask = cumsum <= top_p`` shifted right by one, first token always kept);
* renormalise the kept mass and draw from it (``mx.random.categorical``).

The draw itself comes from MLX's RNG, which no other implementation can
reproduce, so parity is defined on the distribution: the kept set and its
renormalised probabilities.  (The reference draws from
``log(masked_probs + 1e-10)``, which leaves every masked token a weight of
1e-10 against the kept mass of 1 — at most V * 1e-10, 1.3e-5 at V = 128256;
here masked tokens have weight 0.)  For a token-for-token check of a sampler that
takes an explicit uniform ``u`` in [0, 1), ``draw`` restates the same
distribution as an inverse-CDF walk over the kept tokens in vocabulary order:
the first token whose cumulative kept mass exceeds ``u * kept_mass``.

Ties: the reference's order among equal probabilities (a descending view of
an ascending argsort) splits a tie at the top-p boundary by index; here every
token whose probability equals the boundary value is kept (the mass strictly
above it decides), which differs only when probabilities are exactly equal at
the boundary.
"""

from __future__ import annotations

import numpy as np


def softmax_t(logits, temperature: float) -> np.ndarray:
    z = np.asarray(logits, dtype=np.float64) / float(temperature)
    z = z - z.max(axis=-1, keepdims=True)
    e = np.exp(z)
    return e / e.sum(axis=-1, keepdims=True)


def kept_mask(probs, top_p: float) -> np.ndarray:
    """Tokens the top-p filter keeps: the mass strictly above a token's
    probability is <= top_p (rows of ``probs`` independently)."""
    p = np.asarray(probs, dtype=np.float64)
    out = np.zeros(p.shape, dtype=bool)
    for b in range(p.shape[0]):
        order = np.argsort(-p[b], kind="stable")
        sp = p[b][order]
        # mass strictly above each distinct value
        above = np.concatenate([[0.0], np.cumsum(sp)[:-1]])
        # for tied values, the mass strictly above is that of the first of the tie
        first = np.concatenate([[True], sp[1:] != sp[:-1]])
        idx = np.maximum.accumulate(np.where(first, np.arange(sp.size), 0))
        keep_sorted = above[idx] <= top_p
        keep_sorted[0] = True
        out[b][order] = keep_sorted
    return out


def kept_distribution(logits, temperature: float, top_p: float) -> np.ndarray:
    """The renormalised kept distribution, ``[B, V]``."""
    p = softmax_t(logits, temperature)
    k = kept_mask(p, top_p)
    q = np.where(k, p, 0.0)
    return q / q.sum(axis=-1, keepdims=True)


def draw(logits, temperature: float, top_p: float, u) -> np.ndarray:
    """Token per row for uniforms ``u`` (inverse CDF over kept tokens in vocab order)."""
    q = kept_distribution(logits, temperature, top_p)
    u = np.asarray(u, dtype=np.float64).reshape(-1)
    out = np.empty(q.shape[0], dtype=np.int64)
    for b in range(q.shape[0]):
        c = np.cumsum(q[b])
        i = int(np.searchsorted(c, u[b] * c[-1], side="right"))
        kept = np.flatnonzero(q[b] > 0)
        out[b] = min(max(i, kept[0]), kept[-1])
    return out
