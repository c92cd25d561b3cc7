"""k_thread (one thread per output pixel, narrow conv layers) against the
oracle: every layer map bit-identical with k_thread on, with the layer forced
back to k_dense, and through a counting pass (which runs the layer on
k_dense for the reference's fetched-synapse accounting)."""
import numpy as np
import pytest

from helpers import bits_equal

pytestmark = pytest.mark.gpu


def _t(x, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def _np(t):
    return t.detach().cpu().numpy()


def _sync():
    import torch
    torch.cuda.synchronize()


def _narrow_nets():
    from vdttfs import nets
    c, f = nets._conv, nets._fc
    # task-2 semantics (stagger 40, (T+1)-entry LUT by clamp((int)t_in)),
    # K = 3 same-pad convs with 1 to 16 outputs and a 1x1 conv
    vgg_like = nets.NetSpec(
        "narrow_vgg", 9, 7, 3,
        (c(3, 16, 3, nets.PAD_SAME), c(16, 9, 1, nets.PAD_SAME), c(9, 1, 3, nets.PAD_SAME, True),
         f(12, 10, nets.OUT_VMEM)),
        T=40, delta=4, tfs=40.0, lut_mode=nets.LUT_BY_TIN, decay_len=41,
        readout=nets.READ_ARGMAX, tc_in=34.75016403198242, encoder=nets.ENC_LINEAR)
    # task-1 semantics, odd T, 5x5 valid convs of width 5 and 16
    lenet_like = nets.NetSpec(
        "narrow_lenet", 20, 17, 1,
        (c(1, 5, 5, nets.PAD_VALID), c(5, 16, 2, nets.PAD_VALID, True), f(16 * 7 * 6, 10)),
        T=37, delta=8, tfs=0.0, lut_mode=nets.LUT_BY_TB, decay_len=37,
        readout=nets.READ_ARGMIN_FIRST, tc_in=17.452274, encoder=nets.ENC_LINEAR)
    # 33 to 255 inputs per pixel (k_thread's per-thread counting sort):
    # task-1 semantics with a 150-input pooled layer, task-2 semantics with
    # 252 inputs (28 channels x 3x3)
    wide_lenet = nets.NetSpec(
        "wide_lenet", 14, 13, 6,
        (c(6, 16, 5, nets.PAD_VALID, True), c(16, 7, 3, nets.PAD_SAME), f(5 * 4 * 7, 10)),
        T=80, delta=16, tfs=0.0, lut_mode=nets.LUT_BY_TB, decay_len=80,
        readout=nets.READ_ARGMIN_FIRST, tc_in=17.452274, encoder=nets.ENC_LINEAR)
    wide_vgg = nets.NetSpec(
        "wide_vgg", 7, 6, 28,
        (c(28, 12, 3, nets.PAD_SAME, True), c(12, 16, 3, nets.PAD_SAME), f(3 * 3 * 16, 10, nets.OUT_VMEM)),
        T=40, delta=4, tfs=40.0, lut_mode=nets.LUT_BY_TIN, decay_len=41,
        readout=nets.READ_ARGMAX, tc_in=34.75016403198242, encoder=nets.ENC_LINEAR)
    return {"narrow_vgg": vgg_like, "narrow_lenet": lenet_like, "wide_lenet": wide_lenet, "wide_vgg": wide_vgg}


def _case(name, B, td=0.0, gains=None):
    from vdttfs import nets, synth
    net = nets.NETS[name]() if name in nets.NETS else _narrow_nets()[name]
    layers = synth.kaiming_layers(net, 1, gains=gains, td=td)
    img = synth.images(1, B, net.in_h, net.in_w, net.in_c, 0.5, stream=9)
    return net, layers, img


CASES = [("lenet5", 64, 0.0, None), ("lenet_ref", 32, 0.0, None),
         ("narrow_vgg", 6, 0.0, [1.5, 1.5, 2.0, 1.0]), ("narrow_vgg", 5, 3.0, [1.5, 1.5, 2.0, 1.0]),
         ("narrow_lenet", 7, 0.0, [0.8, 1.2, 1.0]), ("narrow_lenet", 3, 2.0, [0.8, 1.2, 1.0]),
         ("wide_lenet", 5, 0.0, [1.0, 1.2, 1.0]), ("wide_lenet", 4, 3.0, [1.0, 1.2, 1.0]),
         ("wide_vgg", 4, 0.0, [1.0, 1.2, 1.0]), ("wide_vgg", 3, 2.0, [1.0, 1.2, 1.0])]


@pytest.mark.parametrize("name,B,td,gains", CASES, ids=[f"{c[0]}-B{c[1]}-td{c[2]}" for c in CASES])
def test_thread_integrator_bitexact(O, dev, name, B, td, gains):
    from vdttfs import engine as E
    net, layers, img = _case(name, B, td, gains)
    spikes = O.encode_linear(img, net.T) if net.encoder == 2 else O.encode_log(img, net.tc_in, net.td_in, net.T)
    ref = O.run_net(net, layers, spikes, keep=True)
    m = E.Model(net, layers, lut_source=E.LUT_HOST_LIBM)
    ctx = E.Context(m, B)
    kinds = ctx.layer_kernels()
    thread_layers = [i for i, k in enumerate(kinds) if k == E.KERNEL_THREAD]
    assert thread_layers, f"no layer of {name} runs k_thread: {kinds}"
    if name.startswith("wide"):
        assert thread_layers[:2] == [0, 1], kinds

    def check(tag):
        maps, out, pred = ctx.trace(_t(spikes, dev))
        _sync()
        ri = 0
        for li, l in enumerate(net.layers):
            assert bits_equal(_np(maps[li]).reshape(-1), ref["maps"][ri]), f"{tag}: layer {li} differs"
            ri += 2 if l.pool_after else 1
        assert bits_equal(_np(out), ref["out"]) and np.array_equal(_np(pred), ref["pred"]), tag

    check("k_thread")
    fired = np.mean(ref["maps"][0] < net.inf_time)
    assert 0.0 < fired < 1.0, f"first layer fired fraction {fired}: the case tests nothing"
    out_h, pred_h = ctx.infer(_t(spikes, dev))      # graph path
    _sync()
    assert bits_equal(_np(out_h), ref["out"]) and np.array_equal(_np(pred_h), ref["pred"])
    ctx.set_counting(True)
    check("counting")
    events, fetched = ctx.counters()
    assert events == sum(ref["events"]) and fetched == sum(ref["fetched"])
    ctx.set_counting(False)
    for li in thread_layers:
        ctx.set_layer_kernel(li, E.KERNEL_DENSE)
    check("forced k_dense")
    ctx.close()
    m.close()


def test_thread_kernel_rejected_where_unsupported(O, dev):
    """VGG-16's layers are all too wide (C_out >= 64) or have too many inputs
    per pixel for k_thread; forcing it is VDT_ERR_UNSUPPORTED."""
    from vdttfs import engine as E, nets, synth
    net = nets.vgg16()
    m = E.Model(net, synth.kaiming_layers(net, 3), lut_source=E.LUT_HOST_LIBM)
    ctx = E.Context(m, 2)
    assert E.KERNEL_THREAD not in ctx.layer_kernels()
    for li in range(len(net.layers)):
        with pytest.raises(E.VdtError) as ei:
            ctx.set_layer_kernel(li, E.KERNEL_THREAD)
        assert ei.value.status == 5
    ctx.close()
    m.close()


PAIR_CASES = [(1, 3), (7, 5), (16, 3), (17, 3), (10, 1)]


@pytest.mark.parametrize("c_out,B", PAIR_CASES, ids=[f"cout{c}-B{b}" for c, b in PAIR_CASES])
def test_dense_two_pixels_per_warp_bitexact(O, dev, c_out, B):
    """k_dense with at most 16 output channels runs two pixels per warp
    (k_dense_pair) outside counting passes: odd pixel counts (the last warp
    holds one pixel), 1 to 16 channels, and 17 channels (one pixel per warp)
    give the oracle's maps bit for bit, with and without counting.  Layers
    this narrow run k_thread by default, so k_dense is chosen explicitly."""
    from vdttfs import engine as E, nets, synth
    c, f = nets._conv, nets._fc
    net = nets.NetSpec(
        "pair", 7, 9, 8, (c(8, c_out, 3, nets.PAD_SAME), f(7 * 9 * c_out, 10, nets.OUT_VMEM)),
        T=40, delta=8, tfs=40.0, lut_mode=nets.LUT_BY_TIN, decay_len=41,
        readout=nets.READ_ARGMAX, tc_in=34.75016403198242, encoder=nets.ENC_LINEAR)
    layers = synth.kaiming_layers(net, 1, gains=[1.6, 1.0])
    img = synth.images(1, B, 7, 9, 8, 0.3, stream=11)
    spikes = O.encode_linear(img, net.T)
    ref = O.run_net(net, layers, spikes, keep=True)
    assert 0.0 < np.mean(ref["maps"][0] < net.inf_time) < 1.0
    m = E.Model(net, layers, lut_source=E.LUT_HOST_LIBM)
    ctx = E.Context(m, B)
    assert ctx.layer_kernels()[0] == (E.KERNEL_THREAD if c_out <= 16 else E.KERNEL_DENSE)
    ctx.set_layer_kernel(0, E.KERNEL_DENSE)
    for counting in (False, True):
        ctx.set_counting(counting)
        maps, out, pred = ctx.trace(_t(spikes, dev))
        _sync()
        assert bits_equal(_np(maps[0]).reshape(-1), ref["maps"][0]), f"counting={counting}"
        assert bits_equal(_np(out), ref["out"]) and np.array_equal(_np(pred), ref["pred"])
    ctx.close()
    m.close()
