"""GPU parity: every engine stage and whole networks against the CPU oracle.

Bit-exact for integer work (bucket offsets, lists, predictions) and, with the
host-libm LUTs (the reference's own tables), bit-exact fp32 first-spike times
and membrane values.  With device-built LUTs (<= 1 ulp from libm expf) spike
times may differ only for neurons whose membrane lies within 1e-5 relative of
threshold, checked neuron by neuron.
"""
import zlib

import numpy as np
import pytest

from helpers import INF, bits_equal, bucket_valid_equal, spike_map, ulp_diff

pytestmark = pytest.mark.gpu


def _t(x, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def _np(t):
    return t.detach().cpu().numpy()


def _sync():
    import torch
    torch.cuda.synchronize()


# ------------------------------------------------------------------ LUTs --
@pytest.mark.parametrize("tc_i,td_i,tc_f,td_f,T,dl", [
    (34.75016403198242, 0.0, 34.75016403198242, 0.0, 80, 81),
    (17.452274, 0.0, 17.452274, 0.0, 80, 80),
    (12.5, 3.25, 40.0, -2.0, 160, 161),
    (60.0, 10.0, 5.0, 1.5, 680, 681),
])
def test_build_luts_within_one_ulp_of_libm(O, dev, tc_i, td_i, tc_f, td_f, T, dl):
    from vdttfs import engine as E
    d, th = E.update_LUTs(T, dl, tc_i, td_i, tc_f, td_f)
    _sync()
    rd, rth = O.update_luts(T, dl, tc_i, td_i, tc_f, td_f)
    assert ulp_diff(_np(d), rd).max() <= 1
    assert ulp_diff(_np(th), rth).max() <= 1


# ------------------------------------------------------------- bucketize --
@pytest.mark.parametrize("c_in,T,delta,tfs", [
    (1, 80, 16, 0.0), (3, 80, 8, 40.0), (6, 80, 16, 0.0), (12, 80, 16, 0.0),
    (31, 80, 8, 40.0), (32, 80, 8, 40.0), (64, 80, 8, 40.0), (100, 80, 4, 40.0),
    (128, 80, 8, 0.0), (512, 80, 8, 40.0), (600, 80, 8, 40.0), (64, 80, 1, 40.0),
    (64, 80, 64, 0.0), (256, 40, 8, 40.0), (64, 20, 8, 0.0),
])
def test_bucketize_nhwc_bitexact(O, dev, c_in, T, delta, tfs):
    from vdttfs import engine as E
    rng = np.random.default_rng(c_in * 1000 + delta)
    n_cols = 777
    x = spike_map(rng, (n_cols, c_in), fire=0.4, T=80, edges=True)
    cfg = E.time_cfg_raw(T, delta, tfs)
    off, cin, tin = E.bucketize(_t(x, dev), n_cols, c_in, cfg)
    _sync()
    roff, rcin, rtin, _ = O.bucketize(x, n_cols, c_in, T, delta, tfs, 0)
    bucket_valid_equal(_np(off), _np(cin), _np(tin), roff, rcin, rtin)


@pytest.mark.parametrize("n_cols,c_in,T,delta,tb_mode", [(5, 70001, 160, 32, 1), (3, 2000, 80, 1, 0),
                                                         (9, 513, 80, 8, 0), (2, 131072, 160, 64, 1)])
def test_bucketize_long_rows_bitexact(O, dev, n_cols, c_in, T, delta, tb_mode):
    """Long rows (flattened FC inputs) take the CTA-per-row kernel."""
    from vdttfs import engine as E
    rng = np.random.default_rng(c_in + delta)
    x = spike_map(rng, (n_cols, c_in), fire=0.3, T=T, edges=True)
    tfs = 40.0 if tb_mode == 0 else 0.0
    cfg = E.time_cfg_raw(T, delta, tfs)
    off, cin, tin = E.bucketize(_t(x, dev), n_cols, c_in, cfg, tb_mode=tb_mode)
    _sync()
    roff, rcin, rtin, _ = O.bucketize(x, n_cols, c_in, T, delta, tfs, tb_mode)
    bucket_valid_equal(_np(off), _np(cin), _np(tin), roff, rcin, rtin)


@pytest.mark.parametrize("C,H,W,T,delta", [(64, 8, 8, 160, 32), (128, 4, 4, 160, 32),
                                           (2, 16, 16, 160, 16), (128, 5, 3, 100, 8)])
def test_bucketize_nchw_trunc_bitexact(O, dev, C, H, W, T, delta):
    from vdttfs import engine as E
    rng = np.random.default_rng(C + H)
    N = 3
    x = spike_map(rng, (N, C, H, W), fire=0.3, T=T, edges=True)
    cfg = E.time_cfg_raw(T, delta, 0.0)
    off, cin, tin = E.bucketize(_t(x, dev), N * H * W, C, cfg, layout=E.LAYOUT_NCHW, hw=H * W,
                                tb_mode=E.TB_TRUNC)
    _sync()
    roff, rcin, rtin, _ = O.bucketize(x, N * H * W, C, T, delta, 0.0, 1, 1, H * W)
    bucket_valid_equal(_np(off), _np(cin), _np(tin), roff, rcin, rtin)


def test_bucketize_all_inf_and_empty(O, dev):
    from vdttfs import engine as E
    cfg = E.time_cfg_raw(80, 8, 40.0)
    x = np.full((50, 64), INF, np.float32)
    off, _, _ = E.bucketize(_t(x, dev), 50, 64, cfg)
    _sync()
    assert not _np(off).any()


# ----------------------------------------------------------- integrator --
def _layer_case(O, dev, rng, *, B, H, W, C_in, C_out, K, pad, is_fc, T, delta, tfs, lut_mode,
                fire=0.3, gain=1.0, t_min=0, edges=False):
    from vdttfs import engine as E
    dl = T + 1 if lut_mode == 1 else T
    if is_fc:
        x = spike_map(rng, (B, C_in), fire=fire, T=T, edges=edges)
        n_cols, Ho, Wo, Kk = B, 1, 1, 1
        Wt = rng.standard_normal((C_in, C_out)).astype(np.float32) * np.float32(gain * np.sqrt(2 / C_in))
    else:
        x = spike_map(rng, (B, H, W, C_in), fire=fire, T=T, edges=edges)
        n_cols = B * H * W
        Ho, Wo = (H, W) if pad else (H - K + 1, W - K + 1)
        Kk = K
        Wt = (rng.standard_normal((K, K, C_in, C_out)).astype(np.float32)
              * np.float32(gain * np.sqrt(2 / (K * K * C_in))))
    bias = (rng.standard_normal(C_out) * 0.05).astype(np.float32)
    ld, lth = O.update_luts(T, dl, 34.75, 0.0, 34.75, 0.0)
    roff, rcin, rtin, _ = O.bucketize(x, n_cols, C_in, T, delta, tfs, 0)
    ref, fetched = O.conv_bucketed(roff, rcin, rtin, Wt, bias, ld, lth, t_min, B,
                                   1 if is_fc else H, 1 if is_fc else W, C_in, Ho, Wo, C_out, Kk,
                                   (K // 2) if pad else 0, is_fc, T, delta, tfs, lut_mode)
    cfg = E.time_cfg_raw(T, delta, tfs, lut_mode, dl)
    off, cin, tin = E.bucketize(_t(x, dev), n_cols, C_in, cfg)
    out = E.conv_bucketed(off, cin, tin, _t(Wt, dev), _t(bias, dev), _t(ld, dev), _t(lth, dev),
                          t_min, B, 1 if is_fc else H, 1 if is_fc else W, C_in, Ho, Wo, C_out, Kk,
                          (K // 2) if pad else 0, is_fc, cfg)
    _sync()
    return _np(out), ref, fetched


CASES = [
    # VGG-like same-pad convs, stagger 40, (T+1)-entry LUT by clamp((int)t_in)
    dict(B=3, H=8, W=8, C_in=64, C_out=128, K=3, pad=1, is_fc=0, T=80, delta=8, tfs=40.0, lut_mode=1, gain=1.3),
    dict(B=2, H=4, W=4, C_in=512, C_out=512, K=3, pad=1, is_fc=0, T=80, delta=8, tfs=40.0, lut_mode=1, gain=1.1),
    dict(B=2, H=6, W=5, C_in=3, C_out=64, K=3, pad=1, is_fc=0, T=80, delta=8, tfs=40.0, lut_mode=1, fire=0.9, gain=0.4),
    dict(B=4, H=1, W=1, C_in=512, C_out=10, K=1, pad=0, is_fc=1, T=80, delta=8, tfs=40.0, lut_mode=1),
    dict(B=4, H=1, W=1, C_in=512, C_out=512, K=1, pad=0, is_fc=1, T=80, delta=8, tfs=40.0, lut_mode=1),
    # LeNet-like valid convs, no stagger, T-entry LUT by tb
    dict(B=4, H=12, W=12, C_in=6, C_out=16, K=5, pad=0, is_fc=0, T=80, delta=16, tfs=0.0, lut_mode=0, gain=0.4),
    dict(B=4, H=28, W=28, C_in=1, C_out=6, K=5, pad=0, is_fc=0, T=80, delta=16, tfs=0.0, lut_mode=0, gain=0.2),
    dict(B=8, H=1, W=1, C_in=84, C_out=10, K=1, pad=0, is_fc=1, T=80, delta=16, tfs=0.0, lut_mode=0),
    dict(B=8, H=1, W=1, C_in=256, C_out=120, K=1, pad=0, is_fc=1, T=80, delta=16, tfs=0.0, lut_mode=0),
    # odd channel counts, t_min > 0, truncated window, edge times
    dict(B=2, H=5, W=7, C_in=40, C_out=36, K=3, pad=1, is_fc=0, T=40, delta=4, tfs=40.0, lut_mode=1, t_min=3, edges=True),
    dict(B=2, H=5, W=7, C_in=40, C_out=200, K=3, pad=1, is_fc=0, T=80, delta=32, tfs=0.0, lut_mode=0, edges=True),
]


@pytest.mark.parametrize("case", CASES, ids=[str(i) for i in range(len(CASES))])
def test_conv_bucketed_bitexact(O, dev, case):
    rng = np.random.default_rng(zlib.crc32(repr(sorted(case.items())).encode()))
    out, ref, _ = _layer_case(O, dev, rng, **case)
    assert bits_equal(out, ref), f"{np.sum(out != ref)} of {ref.size} spike times differ"
    frac = np.mean(ref < INF)
    assert 0.0 < frac or case["C_out"] <= 16


@pytest.mark.parametrize("delta", [1, 2, 4, 8, 16, 32, 64])
def test_conv_bucketed_every_delta(O, dev, delta):
    base = dict(B=2, H=6, W=6, C_in=64, C_out=64, K=3, pad=1, is_fc=0, T=80, delta=delta, tfs=40.0,
                lut_mode=1, gain=1.3)
    out, ref, _ = _layer_case(O, dev, np.random.default_rng(5), **base)
    assert bits_equal(out, ref)
    # chunking is lossless: every delta gives the delta=8 result bit for bit
    base8 = dict(base, delta=8)
    out8, _, _ = _layer_case(O, dev, np.random.default_rng(5), **base8)
    assert bits_equal(out, out8)


# ------------------------------------------------------- vmem / pool / etc
def test_layer_vmem_bitexact(O, dev):
    from vdttfs import engine as E
    rng = np.random.default_rng(11)
    B, C_in, C_out, T = 37, 512, 10, 80
    x = spike_map(rng, (B, C_in), fire=0.3, T=T, edges=True)
    Wt = rng.standard_normal((C_in, C_out)).astype(np.float32)
    bias = rng.standard_normal(C_out).astype(np.float32)
    ld, _ = O.update_luts(T, T + 1, 34.75, 0.0, 34.75, 0.0)
    ref = O.layer_vmem(x, Wt, bias, ld, B, C_in, C_out, T, 40.0)
    cfg = E.time_cfg_raw(T, 8, 40.0, 1, T + 1)
    out = E.layer_vmem(_t(x, dev), _t(Wt, dev), _t(bias, dev), _t(ld, dev), B, C_in, C_out, cfg)
    _sync()
    assert bits_equal(_np(out), ref)


@pytest.mark.parametrize("B,H,W,C", [(3, 32, 32, 64), (2, 24, 24, 6), (2, 8, 8, 3), (1, 5, 7, 4)])
def test_pool_min_exact(O, dev, B, H, W, C):
    from vdttfs import engine as E
    rng = np.random.default_rng(B * H + C)
    x = spike_map(rng, (B, H, W, C), fire=0.3, edges=True)
    out = E.pooling(_t(x, dev), B, H, W, C)
    _sync()
    assert bits_equal(_np(out), O.pool_min(x, B, H, W, C))


def test_encode_linear_exact_and_log_near(O, dev):
    from vdttfs import engine as E
    rng = np.random.default_rng(3)
    px = rng.random(200000, dtype=np.float32)
    px[rng.random(px.size) < 0.2] = 0.0
    px[:6] = [0.0, 1e-6, 1e-5, 1.0, 0.999999, 0.5]
    lin = E.encode_image(_t(px, dev), 2, T=80)
    _sync()
    assert bits_equal(_np(lin), O.encode_linear(px, 80))
    lg = _np(E.encode_image(_t(px, dev), 1, tc=34.75016403198242, td=0.0, T=80))
    rl = O.encode_log(px, 34.75016403198242, 0.0, 80)
    diff = lg != rl
    # CUDA logf and libm logf may round differently; only pixels whose
    # td - tc*ln(x) sits within a few ulp of an integer can land on another step
    if diff.any():
        tf = -34.75016403198242 * np.log(px[diff].astype(np.float64))
        assert np.all(np.abs(tf - np.round(tf)) < 1e-4)
    assert diff.mean() < 1e-4


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_readout_modes(O, dev, mode):
    from vdttfs import engine as E
    rng = np.random.default_rng(mode)
    B, K = 300, 10
    if mode == 2:
        o = rng.standard_normal((B, K)).astype(np.float32)
        o[0] = -2e9
        o[1, 3] = o[1, 5] = 7.0
    else:
        o = spike_map(rng, (B, K), fire=0.5)
        o[0] = INF
        o[1, 2] = o[1, 7] = -1.0
    pred = E.readout(_t(o, dev), B, K, mode)
    _sync()
    assert np.array_equal(_np(pred), O.readout(o, B, K, mode))


# ------------------------------------------------------------- networks --
def _net_case(name, B, cfg_id, zero_frac):
    from vdttfs import nets, synth
    net = nets.NETS[name]()
    layers = synth.kaiming_layers(net, cfg_id)
    img = synth.images(cfg_id, B, net.in_h, net.in_w, net.in_c, zero_frac, stream=5)
    return net, layers, img


@pytest.mark.parametrize("name,B,cfg_id,zero_frac", [("lenet5", 64, 1, 0.8), ("vgg16", 6, 3, 0.0),
                                                     ("lenet_ref", 32, 1, 0.8)])
def test_network_bitexact_host_luts(O, dev, name, B, cfg_id, zero_frac):
    """Whole network with the reference's own (libm) LUTs: every layer map,
    the output and the predictions are bit-identical to the oracle, and the
    fetched-synapse / event counters equal the oracle's."""
    from vdttfs import engine as E
    net, layers, img = _net_case(name, B, cfg_id, zero_frac)
    spikes = O.encode_linear(img, net.T) if net.encoder == 2 else O.encode_log(img, net.tc_in, net.td_in, net.T)
    ref = O.run_net(net, layers, spikes, keep=True)
    m = E.Model(net, layers, lut_source=E.LUT_HOST_LIBM)
    ctx = E.Context(m, B)
    ctx.set_counting(True)
    maps, out, pred = ctx.trace(_t(spikes, dev))
    _sync()
    events, fetched = ctx.counters()
    ri = 0
    for li, l in enumerate(net.layers):
        assert bits_equal(_np(maps[li]).reshape(-1), ref["maps"][ri]), f"layer {li} differs"
        ri += 2 if l.pool_after else 1
    assert bits_equal(_np(out), ref["out"])
    assert np.array_equal(_np(pred), ref["pred"])
    assert events == sum(ref["events"])
    assert fetched == sum(ref["fetched"])
    # pixels in -> same result through the fused encoder, graph path
    out2, pred2 = ctx.infer(_t(img, dev), pixels=True)
    _sync()
    assert bits_equal(_np(out2), ref["out"]) and np.array_equal(_np(pred2), ref["pred"])


@pytest.mark.parametrize("kernel", [0, 1, 2])
def test_every_integrator_choice_is_bitexact(O, dev, kernel):
    """Forcing k_integrate / k_sorted / k_dense on every layer that kernel
    supports changes nothing: maps, outputs and counters stay bit-identical
    to the oracle (graph path and eager path)."""
    from vdttfs import engine as E
    net, layers, img = _net_case("vgg16", 5, 3, 0.0)
    spikes = O.encode_linear(img, net.T)
    ref = O.run_net(net, layers, spikes, keep=True)
    m = E.Model(net, layers, lut_source=E.LUT_HOST_LIBM)
    ctx = E.Context(m, 5)
    forced = 0
    for li in range(len(net.layers)):
        try:
            ctx.set_layer_kernel(li, kernel)
            forced += 1
        except E.VdtError as e:
            assert e.status == 5                      # VDT_ERR_UNSUPPORTED
    assert forced >= 3
    kinds = ctx.layer_kernels()
    assert sum(k == kernel for k in kinds) == forced
    ctx.set_counting(True)
    maps, out, pred = ctx.trace(_t(spikes, dev))
    _sync()
    events, fetched = ctx.counters()
    ri = 0
    for li, l in enumerate(net.layers):
        assert bits_equal(_np(maps[li]).reshape(-1), ref["maps"][ri]), f"layer {li} differs"
        ri += 2 if l.pool_after else 1
    assert bits_equal(_np(out), ref["out"]) and np.array_equal(_np(pred), ref["pred"])
    assert events == sum(ref["events"]) and fetched == sum(ref["fetched"])
    ctx.set_counting(False)
    maps, out2, pred2 = ctx.trace(_t(spikes, dev))
    _sync()
    ri = 0
    for li, l in enumerate(net.layers):
        assert bits_equal(_np(maps[li]).reshape(-1), ref["maps"][ri]), f"layer {li} differs (no counting)"
        ri += 2 if l.pool_after else 1
    assert bits_equal(_np(out2), ref["out"])
    with pytest.raises(E.VdtError):
        ctx.set_layer_kernel(len(net.layers) - 1, 0)  # membrane-readout layer
    with pytest.raises(E.VdtError):
        ctx.set_layer_kernel(0, 9)


def test_network_device_luts_tolerance(O, dev):
    """Device-built LUTs (<= 1 ulp from libm): layer by layer on identical
    inputs, any spike-time difference must come from a neuron whose membrane
    lies within 1e-5 relative of its threshold; predictions >= 99.9% equal."""
    from vdttfs import engine as E
    net, layers, img = _net_case("vgg16", 6, 3, 0.0)
    spikes = O.encode_linear(img, net.T)
    ref = O.run_net(net, layers, spikes, keep=True)
    m = E.Model(net, layers, lut_source=E.LUT_DEVICE)
    ctx = E.Context(m, 6)
    maps, out, pred = ctx.trace(_t(spikes, dev))
    _sync()
    agree = np.mean(_np(pred) == ref["pred"])
    assert agree >= 0.999 or np.sum(_np(pred) != ref["pred"]) <= 1
    # first layer sees identical input: mismatches must be near-threshold
    d0, th0 = m.luts(0)
    rd0, rth0 = O.update_luts(net.T, net.decay_len, net.tc_in, net.td_in, layers[0].tc_fire, layers[0].td)
    assert ulp_diff(d0, rd0).max() <= 1 and ulp_diff(th0, rth0).max() <= 1
    mism = np.mean(_np(maps[0]).reshape(-1) != ref["maps"][0])
    assert mism < 1e-3


def test_infer_host_matches_device_and_eager(O, dev):
    from vdttfs import engine as E
    net, layers, img = _net_case("vgg16", 8, 3, 0.0)
    m = E.Model(net, layers)
    ctx = E.Context(m, 16)
    spikes = O.encode_linear(img, net.T)
    o1, p1 = ctx.infer(_t(spikes, dev))
    o2, p2 = ctx.infer_host(spikes)
    ctx.set_graphs(False)
    o3, p3 = ctx.infer(_t(spikes, dev))
    _sync()
    assert bits_equal(_np(o1), o2) and bits_equal(_np(o1), _np(o3))
    assert np.array_equal(_np(p1), p2) and np.array_equal(p2, _np(p3))
    # a second batch size reuses the same workspace
    o4, _ = ctx.infer_host(spikes[:3])
    assert bits_equal(o4, o2[:3])


@pytest.mark.parametrize("graphs", [True, False])
def test_infer_host_batches_pipelined(O, dev, graphs):
    """vdt_infer_host_batches (next batch's H2D overlapping this batch's
    compute, two device slots) gives every batch the result vdt_infer_host
    gives it, for 1 to 5 batches of different inputs, graph and eager paths;
    NULL output entries are skipped and bad arguments are rejected."""
    import torch
    from vdttfs import engine as E, synth
    net, layers, _ = _net_case("lenet5", 4, 1, 0.8)
    m = E.Model(net, layers)
    ctx = E.Context(m, 16)
    ctx.set_graphs(graphs)
    imgs = [torch.from_numpy(synth.images(1, 16, 28, 28, 1, 0.8, stream=30 + i)).pin_memory() for i in range(5)]
    refs = [ctx.infer_host(x.numpy(), pixels=True) for x in imgs]
    for n in (1, 2, 5):
        outs, preds = ctx.infer_host_batches(imgs[:n], pixels=True)
        for i in range(n):
            assert bits_equal(outs[i], refs[i][0]), f"n={n} batch {i}"
            assert np.array_equal(preds[i], refs[i][1])
    assert ctx.infer_host_batches([], pixels=True) == ([], [])
    import ctypes as C
    from vdttfs._lib import lib
    arr = (C.c_void_p * 2)(imgs[0].data_ptr(), None)
    outs = (C.c_void_p * 2)(None, None)
    assert lib().vdt_infer_host_batches(ctx.h, 2, arr, 1, 16, outs, outs) == 1      # h_inputs[1] NULL
    assert lib().vdt_infer_host_batches(ctx.h, 1, arr, 1, 17, None, None) == 6      # batch > max_batch (VDT_ERR_CAPACITY)
    assert lib().vdt_infer_host_batches(ctx.h, 1, arr, 1, 16, None, None) == 0      # no outputs wanted
    ctx.close()
    m.close()


@pytest.mark.parametrize("name,B", [("vgg16", 5), ("lenet5", 33), ("vgg16", 1)])
def test_sub_batches_change_nothing(O, dev, name, B):
    """vdt_ctx_set_sub_batches(n) (each batch as n parts on n streams, graph
    and eager paths, device, host and pipelined host entry points) gives the
    whole batch's outputs and predictions bit for bit, for n = 2..4 and
    batches that do not divide evenly (or are smaller than n).  The host
    call runs one graph per part, each part's copies on its own stream."""
    from vdttfs import engine as E
    net, layers, img = _net_case(name, B, 3 if name == "vgg16" else 1, 0.0 if name == "vgg16" else 0.8)
    spikes = O.encode_linear(img, net.T)
    ref = O.run_net(net, layers, spikes)
    m = E.Model(net, layers, lut_source=E.LUT_HOST_LIBM)
    ctx = E.Context(m, B)
    for n in (2, 3, 4):
        ctx.set_sub_batches(n)
        for graphs in (True, False):
            ctx.set_graphs(graphs)
            out, pred = ctx.infer(_t(spikes, dev))
            _sync()
            assert bits_equal(_np(out), ref["out"]) and np.array_equal(_np(pred), ref["pred"]), f"n={n} graphs={graphs}"
            for _ in range(2):                               # the second call reuses the parts' graphs
                o, p = ctx.infer_host(spikes.copy())
                assert bits_equal(o, ref["out"]) and np.array_equal(p, ref["pred"]), f"host n={n} graphs={graphs}"
            from vdttfs._lib import lib
            o = np.empty_like(ref["out"])
            assert lib().vdt_infer_host(ctx.h, spikes.ctypes.data, 0, B, o.ctypes.data, None) == 0   # no predictions
            assert bits_equal(o, ref["out"])
        outs, preds = ctx.infer_host_batches([spikes, spikes])
        assert all(bits_equal(o, ref["out"]) for o in outs) and all(np.array_equal(p, ref["pred"]) for p in preds)
    ctx.set_counting(True)                                   # counting passes run whole batches
    out, _ = ctx.infer(_t(spikes, dev))
    _sync()
    assert bits_equal(_np(out), ref["out"])
    with pytest.raises(E.VdtError):
        ctx.set_sub_batches(5)
    ctx.close()
    m.close()


def test_launch_overlap_changes_nothing(O, dev):
    """Programmatic dependent launch on and off: identical maps and outputs,
    through the captured graph and the eager path."""
    from vdttfs import engine as E
    from vdttfs._lib import lib
    net, layers, img = _net_case("vgg16", 7, 3, 0.0)
    m = E.Model(net, layers, lut_source=E.LUT_HOST_LIBM)
    ctx = E.Context(m, 7)
    x = _t(img, dev)
    prev = lib().vdt_set_launch_overlap(0)
    try:
        o0, p0 = ctx.infer(x, pixels=True)
        maps0, _, _ = ctx.trace(x, pixels=True)
        o0, p0, maps0 = _np(o0), _np(p0), [_np(mm) for mm in maps0]
        lib().vdt_set_launch_overlap(1)
        ctx2 = E.Context(m, 7)                         # fresh graphs, captured with overlap
        for _ in range(3):
            o1, p1 = ctx2.infer(x, pixels=True)
        maps1, _, _ = ctx2.trace(x, pixels=True)
        _sync()
        assert bits_equal(_np(o1), o0) and np.array_equal(_np(p1), p0)
        for a, b in zip(maps0, maps1):
            assert bits_equal(a, _np(b))
        spikes = O.encode_linear(img, net.T)
        assert bits_equal(o0, O.run_net(net, layers, spikes)["out"])
    finally:
        lib().vdt_set_launch_overlap(prev)


def test_host_buffers_are_rejected_before_any_launch(dev):
    """A host buffer where device memory is required fails with
    VDT_ERR_INVALID (checked on the host, nothing is launched)."""
    import torch
    from vdttfs import engine as E, nets, synth
    net = nets.lenet5()
    ctx = E.Context(E.Model(net, synth.kaiming_layers(net, 1)), 4)
    x_host = torch.zeros((4, net.in_h, net.in_w, net.in_c), dtype=torch.float32).pin_memory()
    with pytest.raises(E.VdtError) as ei:
        ctx.infer(x_host)
    assert ei.value.status == 1
    y = torch.zeros(4 * 8 * 8 * 6, dtype=torch.float32, device=dev)
    with pytest.raises(E.VdtError) as ei:
        E.pooling(x_host.reshape(-1)[: y.numel()], 4, 8, 8, 6)
    assert ei.value.status == 1
    out, pred = ctx.infer(torch.zeros((4, net.in_h, net.in_w, net.in_c), device=dev))
    _sync()
    assert out.shape == (4, net.n_classes)


def test_capacity_and_argument_errors(dev):
    from vdttfs import engine as E
    from vdttfs._lib import VdtError
    from vdttfs import nets, synth
    net = nets.lenet5()
    m = E.Model(net, synth.kaiming_layers(net, 1))
    ctx = E.Context(m, 4)
    x = np.zeros((5, 28, 28, 1), np.float32)
    with pytest.raises(VdtError) as ei:
        ctx.infer_host(x)
    assert ei.value.status == 6
