"""Shared input generators and comparison helpers for the tests."""
import numpy as np

INF = np.float32(9999.0)

# spike-time values that sit on every branch of the bucket / LUT index rules:
# negative, fractional, the stagger edge 40/41, the window edge T-1 / T, far
# past the window, and INF.
EDGE_TIMES = np.array([0.0, 0.5, 1.0, 7.0, 8.0, 39.0, 39.5, 40.0, 40.5, 41.0, 47.0, 48.0,
                       79.0, 79.5, 80.0, 81.0, 119.0, 120.0, 121.0, 200.0, -0.5, -1.0, -3.0,
                       9998.0, 9999.0, 1e6], np.float32)


def spike_map(rng, shape, fire=0.3, T=80, edges=False):
    """Integer spike times uniform in [0, T) for a `fire` fraction of entries,
    INF elsewhere; with edges, ~10% of entries take EDGE_TIMES values."""
    x = np.where(rng.random(shape) < fire, rng.integers(0, T, shape).astype(np.float32), INF)
    x = x.astype(np.float32)
    if edges:
        m = rng.random(shape) < 0.1
        x[m] = rng.choice(EDGE_TIMES, size=int(m.sum()))
    return x


def bucket_valid_equal(off_a, cin_a, tin_a, off_b, cin_b, tin_b):
    """Compare two bucket sets: offsets exactly, and the first off[:, -1]
    entries of each column's cin/tin lists (the rest is undefined)."""
    assert np.array_equal(off_a, off_b), "offsets differ"
    n = off_a[:, -1]
    mask = np.arange(cin_a.shape[1])[None, :] < n[:, None]
    assert np.array_equal(cin_a[mask], cin_b[mask]), "cin lists differ"
    assert np.array_equal(tin_a[mask].view(np.int32), tin_b[mask].view(np.int32)), "tin lists differ"


def bits_equal(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.int32), b.view(np.int32))


def ulp_diff(a, b):
    a = np.ascontiguousarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.ascontiguousarray(b, np.float32).view(np.int32).astype(np.int64)
    return np.abs(a - b)
