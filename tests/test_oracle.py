"""CPU tests of the oracle itself: hand-computed known answers for every rule
of the reference kernels, and the properties the method guarantees
(lossless, permutation-invariant bucketing; delta-invariant integration)."""
import math

import numpy as np
import pytest

from helpers import INF, bits_equal, spike_map


def test_luts_are_libm_expf(O):
    d, th = O.update_luts(80, 81, 34.75016403198242, 0.0, 17.5, 2.0, 1.0)
    assert d.shape == (81,) and th.shape == (80,)
    for t in (0, 1, 40, 80):
        x = np.float32(-(np.float32(t) - np.float32(0.0)) / np.float32(34.75016403198242))
        assert abs(int(np.float32(math.exp(x)).view(np.int32)) - int(d[t].view(np.int32))) <= 1
    assert d[0] == 1.0
    assert th[2] == 1.0  # t == td_fire


def test_bucketize_known_answer_task2_rules(O):
    # T=80, delta=8, TFS=40: tb = max(0, floor(t - 40)), kept iff tb < 80
    col = np.array([[INF, 0, 45, 41, 40.5, 80, 120, 121, 47.9, 48]], np.float32)
    off, cin, tin, n = O.bucketize(col, 1, 10, 80, 8, 40.0, 0)
    assert n == 7
    assert off[0].tolist() == [0, 5, 6, 6, 6, 6, 7, 7, 7, 7, 7]
    assert cin[0, :7].tolist() == [1, 2, 3, 4, 8, 9, 5]
    assert np.array_equal(tin[0, :7], np.array([0, 45, 41, 40.5, 47.9, 48, 80], np.float32))


def test_bucketize_known_answer_task3_rules(O):
    # tb = (int)t, kept iff 0 <= tb < T  (T=160, delta=32)
    col = np.array([[-0.5, -1.0, 0, 31.9, 32, 159.9, 160, INF]], np.float32)
    off, cin, tin, n = O.bucketize(col, 1, 8, 160, 32, 0.0, 1)
    assert n == 5                                   # -0.5 truncates to 0; -1 and 160 dropped
    assert off[0].tolist() == [0, 3, 4, 4, 4, 5]
    assert cin[0, :5].tolist() == [0, 2, 3, 4, 5]


def test_bucketize_nchw_matches_transposed_nhwc(O):
    rng = np.random.default_rng(1)
    x = spike_map(rng, (2, 16, 3, 5), T=80)                       # NCHW
    a = O.bucketize(x, 2 * 15, 16, 80, 16, 0.0, 1, 1, 15)
    b = O.bucketize(np.ascontiguousarray(x.transpose(0, 2, 3, 1)), 30, 16, 80, 16, 0.0, 1, 0, 1)
    for u, v in zip(a[:3], b[:3]):
        assert np.array_equal(u, v)


@pytest.mark.parametrize("delta", [1, 3, 8, 16, 64])
def test_bucketize_lossless_and_stable(O, delta):
    rng = np.random.default_rng(delta)
    x = spike_map(rng, (200, 37), fire=0.5, T=80, edges=True)
    off, cin, tin, n = O.bucketize(x, 200, 37, 80, delta, 40.0, 0)
    for c in range(200):
        keep = [(i, t) for i, t in enumerate(x[c])
                if t < INF and max(0, math.floor(t - 40.0)) < 80]
        got = list(zip(cin[c, :off[c, -1]].tolist(), tin[c, :off[c, -1]].tolist()))
        assert sorted(got) == sorted(keep)                      # lossless
        nc = (80 + delta - 1) // delta
        for ch in range(nc):
            seg = cin[c, off[c, ch]:off[c, ch + 1]]
            assert np.all(np.diff(seg) > 0)                     # stable (channel order)
            for i in seg:
                assert max(0, math.floor(x[c, i] - 40.0)) // delta == ch


def _one_neuron(O, events, w, bias, lut_d, lut_th, T=80, delta=16, tfs=0.0, lut_mode=0, t_min=0):
    """FC layer with one output neuron and len(w) inputs."""
    x = np.full((1, len(w)), INF, np.float32)
    for ch, t in events:
        x[0, ch] = t
    off, cin, tin, _ = O.bucketize(x, 1, len(w), T, delta, tfs, 0)
    out, fetched = O.conv_bucketed(off, cin, tin, np.asarray(w, np.float32).reshape(-1, 1),
                                   np.array([bias], np.float32), lut_d, lut_th, t_min, 1, 1, 1,
                                   len(w), 1, 1, 1, 1, 0, 1, T, delta, tfs, lut_mode)
    return float(out[0]), fetched


def test_integrator_known_answers(O):
    ones = np.ones(81, np.float32)
    half = np.full(80, 0.5, np.float32)
    # a single event reaching threshold exactly fires (>=) at its arrival
    assert _one_neuron(O, [(0, 3.0)], [0.5], 0.0, ones, half)[0] == 3.0
    # just below threshold never fires
    below = np.nextafter(np.float32(0.5), np.float32(0))
    assert _one_neuron(O, [(0, 3.0)], [below], 0.0, ones, half)[0] == 9999.0
    # two events accumulate in arrival order; firing waits for the second
    assert _one_neuron(O, [(0, 2.0), (1, 21.0)], [0.25, 0.25], 0.0, ones, half)[0] == 21.0
    # bias alone fires at t_min; a threshold below 1e-5 never fires
    assert _one_neuron(O, [], [0.1], 0.6, ones, half, t_min=5)[0] == 5.0
    tiny = np.full(80, 5e-6, np.float32)
    assert _one_neuron(O, [(0, 1.0)], [1.0], 0.0, ones, tiny)[0] == 9999.0
    # early exit: after firing in chunk 0 the chunk-1 event is never fetched
    t, fetched = _one_neuron(O, [(0, 1.0), (1, 30.0)], [0.6, 0.6], 0.0, ones, half)
    assert t == 1.0 and fetched == 1
    t, fetched = _one_neuron(O, [(0, 1.0), (1, 30.0)], [0.2, 0.4], 0.0, ones, half)
    assert t == 30.0 and fetched == 2


def test_integrator_task2_t80_uses_last_decay_entry(O):
    # TFS=40: t_in = 80 -> tb = 40 (chunk 5 at delta 8), LUT index clamp(80) = T
    d = np.zeros(81, np.float32)
    d[80] = 1.0
    th = np.full(80, 0.5, np.float32)
    t, _ = _one_neuron(O, [(0, 80.0)], [0.75], 0.0, d, th, T=80, delta=8, tfs=40.0, lut_mode=1)
    assert t == 40.0
    # an input earlier than the stagger collapses into step 0
    d2 = np.ones(81, np.float32)
    t, _ = _one_neuron(O, [(0, 12.0)], [0.75], 0.0, d2, th, T=80, delta=8, tfs=40.0, lut_mode=1)
    assert t == 0.0


@pytest.mark.parametrize("lut_mode,tfs,pad", [(1, 40.0, 1), (0, 0.0, 0)])
def test_integrator_delta_invariant_bitexact(O, lut_mode, tfs, pad):
    rng = np.random.default_rng(7)
    B, H, W, C_in, C_out, K = 2, 7, 6, 24, 20, 3
    x = spike_map(rng, (B, H, W, C_in), fire=0.35, T=80)
    Wt = (rng.standard_normal((K, K, C_in, C_out)) * 0.5).astype(np.float32)
    bias = np.zeros(C_out, np.float32)
    dl = 81 if lut_mode else 80
    ld, lth = O.update_luts(80, dl, 34.75, 0.0, 34.75, 0.0)
    Ho, Wo = (H, W) if pad else (H - K + 1, W - K + 1)
    outs = []
    for delta in (1, 2, 4, 8, 16, 32, 64, 80):
        off, cin, tin, _ = O.bucketize(x, B * H * W, C_in, 80, delta, tfs, 0)
        y, _ = O.conv_bucketed(off, cin, tin, Wt, bias, ld, lth, 0, B, H, W, C_in, Ho, Wo, C_out,
                               K, pad, 0, 80, delta, tfs, lut_mode)
        outs.append(y)
    assert 0.05 < np.mean(outs[0] < INF) < 0.95
    for y in outs[1:]:
        assert bits_equal(y, outs[0])


def test_pool_and_readout_semantics(O):
    x = np.array([[[[3.0], [INF]], [[1.0], [2.0]]]], np.float32)     # [1, 2, 2, 1]
    assert O.pool_min(x, 1, 2, 2, 1).tolist() == [1.0]
    o = np.array([[INF, INF], [5.0, 5.0], [7.0, 2.0]], np.float32)
    assert O.readout(o, 3, 2, 0).tolist() == [-1, 0, 1]              # t1: -1 when nothing fires
    assert O.readout(o, 3, 2, 1).tolist() == [0, 0, 1]               # t3: class 0 start
    v = np.array([[-2e9, -3e9], [1.0, 1.0]], np.float32)
    assert O.readout(v, 2, 2, 2).tolist() == [-1, 0]                 # t2: argmax from -1e9


def test_dvs_pool_single_spike_known_answer(O):
    # one input spike at t: I=1, V accumulates sum_k d^k; th 5, d = exp(-1/5)
    from vdttfs import nets
    spec = nets.dvs_ref()
    x = np.full((1, 1, 2, 2), INF, np.float32)
    x[0, 0, 1, 0] = 10.0
    out = O.dvs_pool(x, 1, 1, 2, 2, spec)
    V, I, fire = np.float32(0), np.float32(0), None
    for t in range(10, 160):
        I = np.float32(I * np.float32(spec.decay_conv) + (1.0 if t == 10 else 0.0))
        V = np.float32(V + I)
        if V >= 5.0:
            fire = t
            break
    assert out[0] == fire


@pytest.mark.parametrize("delta", [8, 16, 32])
def test_dvs_conv_delta_invariant(O, delta):
    from vdttfs import nets
    rng = np.random.default_rng(2)
    spec = nets.dvs_ref(delta=delta)
    x = spike_map(rng, (2, 8, 6, 6), fire=0.4, T=160)
    w = (rng.standard_normal((5, 8, 3, 3)) * 2.0).astype(np.float32)
    y, _, _ = O.dvs_conv(x, w, 2, 8, 5, 6, 6, spec)
    y32, _, _ = O.dvs_conv(x, w, 2, 8, 5, 6, 6, nets.dvs_ref(delta=32))
    assert bits_equal(y, y32)


@pytest.mark.parametrize("delta,tfs", [(4, 40.0), (8, 40.0), (16, 0.0), (32, 0.0), (64, 40.0)])
def test_time_sorted_buckets_refine_the_chunk_buckets(O, delta, tfs):
    """The fused path sorts at delta = 1; its offsets at multiples of delta are
    the reference's chunk offsets, and each chunk holds the same events."""
    rng = np.random.default_rng(delta)
    x = spike_map(rng, (300, 45), fire=0.5, T=80, edges=True)
    off, cin, tin, n = O.bucketize(x, 300, 45, 80, delta, tfs, 0)
    fo, fc, ft, n1 = O.bucketize(x, 300, 45, 80, 1, tfs, 0)
    assert n == n1
    nc = (80 + delta - 1) // delta
    idx = [min(c * delta, 80) for c in range(nc)] + [80]
    assert np.array_equal(off, fo[:, idx])
    for c in range(300):
        for ch in range(nc):
            a, b = off[c, ch], off[c, ch + 1]
            assert sorted(cin[c, a:b]) == sorted(fc[c, a:b])
