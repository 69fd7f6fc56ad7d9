"""Paired batch statistics for comparing two implementations' timings.

Restates the reference's batch-level comparison (bench/stats.py:4-26): the
timings of one shape come in B paired batches (one median per batch and
implementation, the batches run in interleaved order), and the speed-up is the
ratio of the medians of the batch medians.  Its 95 % interval is a block
bootstrap over whole batches: `draws` resamples of B batch indices, each giving
median(base[idx]) / median(candidate[idx]).  The speed-up counts as a WIN when
the whole interval lies above 1.05, a LOSS when it lies below 1/1.05, a TIE
when it lies inside [1/1.05, 1.05], and is UNCERTAIN otherwise or with fewer
than `minimum` batches.  Seed and draw count are the reference's, so the same
batch medians give the same interval.
"""
from __future__ import annotations

import numpy as np

SEED = 20260908
DRAWS = 10000
THRESHOLD = 1.05
MINIMUM_BATCHES = 10


def _positive_vector(values, name):
    a = np.asarray(values, dtype=float)
    if a.ndim != 1 or a.size == 0 or not np.all(np.isfinite(a)) or np.any(a <= 0):
        raise ValueError(f'{name}: finite positive timings required')
    return a


def describe(values):
    """Median, 10th and 90th percentile of positive timings (bench/stats.py:4-9)."""
    a = _positive_vector(values, 'timings')
    return {'median': float(np.median(a)), 'p10': float(np.quantile(a, 0.1)),
            'p90': float(np.quantile(a, 0.9))}


def classify(low, high, threshold=THRESHOLD):
    """WIN / LOSS / TIE / UNCERTAIN from a speed-up interval (bench/stats.py:22-23)."""
    if low > threshold:
        return 'WIN'
    if high < 1 / threshold:
        return 'LOSS'
    if low >= 1 / threshold and high <= threshold:
        return 'TIE'
    return 'UNCERTAIN'


def compare_batches(base, candidate, minimum=MINIMUM_BATCHES, seed=SEED, draws=DRAWS):
    """Speed-up of `candidate` over `base` from paired batch medians
    (bench/stats.py:11-26); both are per-batch medians of one shape."""
    b = _positive_vector(base, 'base')
    c = _positive_vector(candidate, 'candidate')
    if b.size != c.size:
        raise ValueError('paired batches required: base and candidate differ in length')
    speedup = float(np.median(b) / np.median(c))
    n = b.size
    if n < minimum:
        return {'speedup': speedup, 'classification': 'UNCERTAIN', 'ci95': None, 'paired_batches': n,
                'reason': f'confirmation requires {minimum} independent batches'}
    idx = np.random.default_rng(seed).integers(0, n, size=(draws, n))
    ratios = np.median(b[idx], axis=1) / np.median(c[idx], axis=1)
    low, high = (float(q) for q in np.quantile(ratios, [0.025, 0.975]))
    return {'speedup': speedup, 'classification': classify(low, high), 'ci95': [low, high],
            'paired_batches': n, 'method': 'paired batch median block bootstrap', 'draws': draws}
