"""GPU: k_sorted's chunks with more events than its per-warp record buffer
(512 records), integrated slot by slot, against the oracle bit for bit.

Every input here fires inside one k_sorted chunk (8 steps), so a pixel's
chunk holds about 60% of its K*K*C_in inputs: 1,382 events for 3x3x256
inputs.  Both neuron models go through that path: the LIF integrator of
tasks 1-2 (k_conv_bucketed, t2:84-170, via a network layer forced onto
k_sorted) and the task-3 CuLIF one (conv_bucketed_early, t3:109-143, via
vdt_dvs_conv_bucketed at chunk width 8).
"""
import numpy as np
import pytest

from helpers import INF, bits_equal

pytestmark = pytest.mark.gpu

SORTED = 1


def _t(x, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def _np(t):
    import torch
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("tfs,T", [(40.0, 80), (0.0, 37)], ids=["task2", "task1"])
def test_sorted_oversize_chunks_lif(O, dev, tfs, T):
    from vdttfs import engine as E, nets, synth
    task2 = tfs > 0
    net = nets.NetSpec("big", 4, 5, 256, (nets._conv(256, 128, 3, nets.PAD_SAME), nets._fc(4 * 5 * 128, 10)),
                       T=T, delta=8, tfs=tfs, lut_mode=nets.LUT_BY_TIN if task2 else nets.LUT_BY_TB,
                       decay_len=T + 1 if task2 else T, readout=nets.READ_ARGMIN_FIRST,
                       tc_in=34.75016403198242 if task2 else 17.452274, encoder=nets.ENC_LINEAR)
    layers = synth.kaiming_layers(net, 2, gains=[0.25, 1.0])
    rng = np.random.default_rng(5)
    B = 3
    lo = tfs if task2 else 0.0                              # all events in the first k_sorted chunk (8 steps)
    x = np.where(rng.random((B, 4, 5, 256)) < 0.6, np.floor(lo + 8 * rng.random((B, 4, 5, 256))), INF)
    x = x.astype(np.float32)
    ref = O.run_net(net, layers, x, keep=True)
    fired = np.mean(ref["maps"][0] < INF)
    assert 0.0 < fired < 1.0, f"fired fraction {fired}"
    m = E.Model(net, layers, lut_source=E.LUT_HOST_LIBM)
    ctx = E.Context(m, B)
    ctx.set_layer_kernel(0, SORTED)
    maps, out, pred = ctx.trace(_t(x, dev))
    assert bits_equal(_np(maps[0]).reshape(-1), ref["maps"][0])
    assert bits_equal(_np(out), ref["out"]) and np.array_equal(_np(pred), ref["pred"])
    out2, pred2 = ctx.infer(_t(x, dev))                       # graph path
    assert bits_equal(_np(out2), ref["out"])
    ctx.close()
    m.close()


def test_sorted_oversize_chunks_culif(O, dev):
    from vdttfs import dvs, nets
    spec = nets.dvs_ref(delta=8)
    rng = np.random.default_rng(6)
    N, C_in, C_out, H, W = 2, 160, 64, 5, 4
    x = np.where(rng.random((N, C_in, H, W)) < 0.6, np.floor(8 * rng.random((N, C_in, H, W))), INF)
    x = x.astype(np.float32)
    w = (rng.standard_normal((C_out, C_in, 3, 3)) * 0.05).astype(np.float32)
    off, cin, tin, _ = O.bucketize(x, N * H * W, C_in, spec.T, 8, 0.0, 1, 1, H * W)
    assert int(off[:, 1].max()) * 9 > 512                   # chunk 0 of a pixel's nine taps
    ref = np.empty(N * C_out * H * W, np.float32)
    O.lib().orc_dvs_conv(O._i(off), O._i(cin), O._f(tin), O._f(w), N, C_in, C_out, H, W, 3, spec.T, 8,
                         spec.decay_conv, spec.th_conv, O._f(ref))
    b = dvs.bucketize_sites(_t(x, dev), N, C_in, H, W, spec)
    out = dvs.conv_bucketed(b, dvs.oihw_to_hwio(_t(w, dev)), N, C_in, C_out, H, W, spec)
    got = _np(out)
    assert bits_equal(got, ref), f"{np.sum(got != ref)} of {ref.size} differ"
    assert 0.0 < np.mean(ref < INF) < 1.0
