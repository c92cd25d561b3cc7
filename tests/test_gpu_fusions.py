"""GPU: the work on the edges of the integrators, fused or not, against the oracle.

* A layer's 2x2 min pool (k_pooling, t1:164-181 / t2:192-209), fused into
  every integrator that runs the layer: k_thread (a quad of threads) and
  k_dense / k_sorted (an integer min of each output into its pooled cell).
  The pooled layer is the network's last layer here, so the output compared
  bit for bit IS the pooled map, including odd map sizes (the last row /
  column dropped) and every channel width the kernels vectorise differently;
  the traced run writes the unpooled map and pools it in a separate pass.
* The pixel encoder (k_encode_image's log encoder, t1:32-42 / t2:32-42, and
  the linear one): fused into k_dense's read of a first layer (the same
  device function as the separate pass), a separate pass in front of the
  other first-layer integrators (fusing it into k_thread's read measured
  slower).
* The readout (t1:313-315, t2:391-392, t3:295-296) fused into the membrane
  readout layer (k_layer_vmem, t2:172-190), every readout mode.
Host-libm LUTs, so every comparison is bit for bit.
"""
import numpy as np
import pytest

from helpers import bits_equal

pytestmark = pytest.mark.gpu

THREAD, DENSE, SORTED, CHUNK = 4, 2, 1, 0


def _t(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _np(t):
    import torch
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def _pooled_net(h, w, c_in, c_out, k, pad, task2):
    from vdttfs import nets
    conv = nets._conv(c_in, c_out, k, pad, True)
    if task2:
        return nets.NetSpec("pooled2", h, w, c_in, (conv,), T=40, delta=4, tfs=40.0, lut_mode=nets.LUT_BY_TIN,
                            decay_len=41, readout=nets.READ_ARGMIN_FIRST, tc_in=34.75016403198242,
                            encoder=nets.ENC_LINEAR)
    return nets.NetSpec("pooled1", h, w, c_in, (conv,), T=37, delta=8, tfs=0.0, lut_mode=nets.LUT_BY_TB,
                        decay_len=37, readout=nets.READ_ARGMIN_FIRST, tc_in=17.452274, encoder=nets.ENC_LINEAR)


POOL_CASES = [
    # (H, W, C_in, C_out, K, pad, task2, kernel, gain)
    (9, 7, 6, 16, 3, 1, True, THREAD, 1.6),     # k_thread's quad shuffles, odd H and W
    (8, 6, 8, 16, 5, 0, False, THREAD, 1.2),    # valid conv, 4x2 output
    (7, 9, 8, 16, 3, 1, True, DENSE, 1.6),      # one channel per lane
    (7, 9, 16, 64, 3, 1, True, DENSE, 1.4),     # two channels per lane
    (5, 7, 32, 128, 3, 1, True, DENSE, 1.2),    # four channels per lane
    (7, 5, 16, 64, 3, 1, False, SORTED, 1.4),
    (5, 7, 32, 256, 3, 1, True, SORTED, 1.2),   # two channel groups per quad
    (6, 6, 64, 512, 3, 1, True, SORTED, 1.1),   # four channel groups
]


@pytest.mark.parametrize("case", POOL_CASES, ids=[f"{c[7]}-{c[0]}x{c[1]}x{c[2]}-{c[3]}" for c in POOL_CASES])
def test_pooled_last_layer_every_integrator(O, dev, case):
    from vdttfs import engine as E, synth
    H, W, ci, co, k, pad, task2, kernel, gain = case
    from vdttfs import nets
    net = _pooled_net(H, W, ci, co, k, nets.PAD_SAME if pad else nets.PAD_VALID, task2)
    layers = synth.kaiming_layers(net, 1, gains=[gain])
    B = 5
    img = synth.images(1, B, H, W, ci, 0.3, stream=31)
    spikes = O.encode_linear(img, net.T)
    ref = O.run_net(net, layers, spikes, keep=True)
    fired = np.mean(ref["maps"][0] < net.inf_time)
    assert 0.05 < fired < 0.95, f"fired fraction {fired}: the case tests little"
    m = E.Model(net, layers, lut_source=E.LUT_HOST_LIBM)
    ctx = E.Context(m, B)
    ctx.set_layer_kernel(0, kernel)
    for graphs in (True, False):
        ctx.set_graphs(graphs)
        out, pred = ctx.infer(_t(spikes))                # not traced: the pool runs fused
        o = _np(out)
        assert o.shape == (B, (H - (0 if pad else k - 1)) // 2 * ((W - (0 if pad else k - 1)) // 2) * co)
        n_bad = int(np.sum(o.view(np.int32) != ref["out"].view(np.int32)))
        assert n_bad == 0, f"graphs={graphs}: {n_bad} of {o.size} pooled values differ"
        assert np.array_equal(_np(pred), ref["pred"])
    maps, out_t, _ = ctx.trace(_t(spikes))               # traced: the unpooled map, then a pool pass
    assert bits_equal(_np(maps[0]).reshape(-1), ref["maps"][0])
    assert bits_equal(_np(out_t), ref["out"])
    ctx.close()
    m.close()


@pytest.mark.parametrize("encoder", [1, 2], ids=["log", "linear"])
@pytest.mark.parametrize("kernel", [THREAD, DENSE, SORTED, CHUNK])
def test_pixels_through_every_first_layer_integrator(O, dev, encoder, kernel):
    """Pixels in, with every integrator on the first layer: the result equals
    the oracle's encoder followed by the network, and the network fed the
    separately encoded spike times."""
    from vdttfs import engine as E, nets, synth
    net = nets.NetSpec("enc", 10, 9, 3, (nets._conv(3, 16, 3, nets.PAD_SAME), nets._fc(10 * 9 * 16, 10)),
                       T=80, delta=8, tfs=40.0, lut_mode=nets.LUT_BY_TIN, decay_len=81,
                       readout=nets.READ_ARGMIN_FIRST, tc_in=34.75016403198242, encoder=encoder)
    layers = synth.kaiming_layers(net, 3, gains=[1.5, 1.2])
    B = 6
    img = synth.images(3, B, 10, 9, 3, 0.2, stream=33)
    spikes = O.encode_log(img, net.tc_in, net.td_in, net.T) if encoder == 1 else O.encode_linear(img, net.T)
    ref = O.run_net(net, layers, spikes, keep=True)
    m = E.Model(net, layers, lut_source=E.LUT_HOST_LIBM)
    ctx = E.Context(m, B)
    ctx.set_layer_kernel(0, kernel)
    maps, out, pred = ctx.trace(_t(img), pixels=True)
    if encoder == 2:                                     # the linear encoder is exact
        assert bits_equal(_np(maps[0]).reshape(-1), ref["maps"][0])
        assert bits_equal(_np(out), ref["out"]) and np.array_equal(_np(pred), ref["pred"])
    # either encoder: the fused read equals the separate encode pass bit for bit
    enc = E.encode_image(_t(img).reshape(-1), encoder, net.tc_in, net.td_in, net.T).reshape(img.shape)
    maps2, out2, pred2 = ctx.trace(enc, pixels=False)
    assert bits_equal(_np(maps[0]), _np(maps2[0]))
    assert bits_equal(_np(out), _np(out2)) and np.array_equal(_np(pred), _np(pred2))
    o3, p3 = ctx.infer(_t(img), pixels=True)             # graph path
    assert bits_equal(_np(o3), _np(out2)) and np.array_equal(_np(p3), _np(pred2))
    ctx.close()
    m.close()


@pytest.mark.parametrize("readout", [0, 1, 2], ids=["argmin_first", "argmin_lowest", "argmax"])
def test_readout_fused_into_the_membrane_layer(O, dev, readout):
    """The last layer's membrane values and the readout computed in the same
    kernel: predictions equal the oracle's readout of the same values,
    including 40 classes (two per lane) and ties."""
    from vdttfs import engine as E, nets, synth
    net = nets.NetSpec("vm", 4, 4, 8, (nets._conv(8, 16, 3, nets.PAD_SAME), nets._fc(4 * 4 * 16, 40, nets.OUT_VMEM)),
                       T=40, delta=4, tfs=40.0, lut_mode=nets.LUT_BY_TIN, decay_len=41, readout=readout,
                       tc_in=34.75016403198242, encoder=nets.ENC_LINEAR)
    layers = synth.kaiming_layers(net, 2, gains=[1.5, 1.0])
    layers[1].kernel[:, 7] = layers[1].kernel[:, 3]      # two equal classes: a tie on every image
    layers[1].bias[7] = layers[1].bias[3]
    B = 33
    img = synth.images(2, B, 4, 4, 8, 0.3, stream=35)
    spikes = O.encode_linear(img, net.T)
    ref = O.run_net(net, layers, spikes)
    m = E.Model(net, layers, lut_source=E.LUT_HOST_LIBM)
    ctx = E.Context(m, B)
    out, pred = ctx.infer(_t(spikes))
    assert bits_equal(_np(out), ref["out"])
    assert np.array_equal(_np(pred), ref["pred"])
    assert np.array_equal(_np(pred), O.readout(_np(out), B, 40, readout))
    ctx.close()
    m.close()


def test_unpooled_conv_last_layer_output_is_the_whole_map(O, dev):
    """A network ending in a conv layer without a pool outputs that layer's
    whole first-spike map, flattened ([B, H * W * C]), on every path."""
    from vdttfs import engine as E, nets, synth
    net = nets.NetSpec("convout", 6, 5, 4, (nets._conv(4, 24, 3, nets.PAD_SAME),), T=40, delta=4, tfs=40.0,
                       lut_mode=nets.LUT_BY_TIN, decay_len=41, readout=nets.READ_ARGMIN_FIRST,
                       tc_in=34.75016403198242, encoder=nets.ENC_LINEAR)
    assert net.n_classes == 6 * 5 * 24
    layers = synth.kaiming_layers(net, 1, gains=[1.6])
    B = 7
    spikes = O.encode_linear(synth.images(1, B, 6, 5, 4, 0.3, stream=37), net.T)
    ref = O.run_net(net, layers, spikes)
    m = E.Model(net, layers, lut_source=E.LUT_HOST_LIBM)
    assert m.n_classes == net.n_classes
    ctx = E.Context(m, B)
    for kernel in (DENSE, SORTED, CHUNK):
        ctx.set_layer_kernel(0, kernel)
        out, pred = ctx.infer(_t(spikes))
        assert _np(out).shape == (B, net.n_classes)
        assert bits_equal(_np(out), ref["out"]) and np.array_equal(_np(pred), ref["pred"]), f"kernel {kernel}"
        o2, p2 = ctx.infer_host(spikes)
        assert bits_equal(o2, ref["out"]) and np.array_equal(p2, ref["pred"])
    ctx.close()
    m.close()


@pytest.mark.parametrize("kernel", [DENSE, SORTED, CHUNK])
def test_pooled_middle_layer_feeds_the_next(O, dev, kernel):
    """A pooled layer inside the network (odd 7x9 map: the last row and
    column dropped) on each integrator: the next layer reads the pooled map
    the integrator wrote (k_dense / k_sorted fused, the chunk integrator with
    a pool pass), graph and eager paths, with sub-batches, bit for bit."""
    from vdttfs import engine as E, nets, synth
    net = nets.NetSpec("midpool", 7, 9, 16, (nets._conv(16, 64, 3, nets.PAD_SAME, True), nets._conv(64, 32, 3, nets.PAD_SAME),
                                             nets._fc(3 * 4 * 32, 10)),
                       T=40, delta=4, tfs=40.0, lut_mode=nets.LUT_BY_TIN, decay_len=41,
                       readout=nets.READ_ARGMIN_FIRST, tc_in=34.75016403198242, encoder=nets.ENC_LINEAR)
    layers = synth.kaiming_layers(net, 5, gains=[1.4, 1.3, 1.0])
    B = 9
    spikes = O.encode_linear(synth.images(5, B, 7, 9, 16, 0.3, stream=39), net.T)
    ref = O.run_net(net, layers, spikes, keep=True)
    assert 0.05 < np.mean(ref["maps"][1] < net.inf_time) < 0.95     # the pooled map
    assert 0.0 < np.mean(ref["maps"][2] < net.inf_time)             # the next layer fires
    m = E.Model(net, layers, lut_source=E.LUT_HOST_LIBM)
    ctx = E.Context(m, B)
    ctx.set_layer_kernel(0, kernel)
    for sub in (1, 2):
        ctx.set_sub_batches(sub)
        for graphs in (True, False):
            ctx.set_graphs(graphs)
            out, pred = ctx.infer(_t(spikes))
            assert bits_equal(_np(out), ref["out"]), f"sub={sub} graphs={graphs}"
            assert np.array_equal(_np(pred), ref["pred"])
    ctx.close()
    m.close()
