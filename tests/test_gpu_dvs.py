"""Task 3 (DVS gesture, CuLIF) on the GPU: every stage through the C ABI,
bit-exact against the golden maps of the reference's own kernels and against
the CPU oracle (oracle/vdt_oracle.c, orc_dvs_*) on seeded inputs.  Spike times
are integers and the CuLIF arithmetic is a fixed FMA/add sequence, so the
tolerance is zero."""
import os
import sys

import numpy as np
import pytest

from conftest import GOLDEN
from helpers import INF, bits_equal, spike_map

sys.path.insert(0, os.path.join(GOLDEN))
from make_golden import DVS_GAINS  # noqa: E402

pytestmark = pytest.mark.gpu


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _np(t):
    import torch
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def test_dvs_ref_network_matches_the_reference_kernels(dev):
    """The reference's own 2x32x32 DVS network: all seven stage maps equal the
    golden maps produced by the reference's kernels, bit for bit."""
    from vdttfs import dvs, nets, synth
    g = np.load(os.path.join(GOLDEN, "net_dvs_ref.npz"))
    spec = nets.dvs_ref()
    wts = synth.dvs_weights(spec, 4, gains=DVS_GAINS)
    w = dvs.DvsWeights(spec, wts, dev)
    r = dvs.run(spec, w, _t(g["frames"].astype(np.float32), dev), keep=True)
    for i, m in enumerate(r["maps"]):
        assert bits_equal(_np(m).reshape(-1), g[f"map{i}"].astype(np.float32)), f"stage {i} differs"
    ref_out = g["map6"].astype(np.float32).reshape(2, spec.classes)
    want = np.array([np.argmin(o) for o in ref_out])           # lowest index among the minima
    assert np.array_equal(_np(r["pred"]), want)


@pytest.mark.parametrize("delta", [8, 16, 32, 64])
def test_conv_bucketed_early_every_delta(O, dev, delta):
    from vdttfs import dvs, nets
    spec = nets.dvs_ref(delta=delta)
    rng = np.random.default_rng(delta)
    N, C_in, C_out, H, W = 2, 48, 96, 9, 7
    x = spike_map(rng, (N, C_in, H, W), fire=0.35, T=spec.T, edges=True)
    w = (rng.standard_normal((C_out, C_in, 3, 3)) * 0.35).astype(np.float32)
    off, cin, tin, _ = O.bucketize(x, N * H * W, C_in, spec.T, delta, 0.0, 1, 1, H * W)
    ref = np.empty(N * C_out * H * W, np.float32)
    fe = O.lib().orc_dvs_conv(O._i(off), O._i(cin), O._f(tin), O._f(w), N, C_in, C_out, H, W, 3, spec.T, delta,
                              spec.decay_conv, spec.th_conv, O._f(ref))
    assert fe > 0
    b = dvs.bucketize_sites(_t(x, dev), N, C_in, H, W, spec)
    wd = dvs.oihw_to_hwio(_t(w, dev))
    out = dvs.conv_bucketed(b, wd, N, C_in, C_out, H, W, spec)
    got = _np(out)
    assert bits_equal(got, ref), f"{np.sum(got != ref)} of {ref.size} differ"
    assert 0.0 < np.mean(ref < INF) < 1.0
    # NHWC output holds the same values
    out2 = dvs.conv_bucketed(b, wd, N, C_in, C_out, H, W, spec, out_layout=0)
    nhwc = _np(out2).reshape(N, H, W, C_out).transpose(0, 3, 1, 2).reshape(-1)
    assert bits_equal(nhwc, ref)


DENSE_CASES = [(8, 160, 48, 96), (32, 160, 128, 64), (32, 150, 48, 96), (16, 77, 3, 40), (64, 160, 20, 128)]


@pytest.mark.parametrize("delta,T,C_in,C_out", DENSE_CASES, ids=[f"d{c[0]}-T{c[1]}-cin{c[2]}" for c in DENSE_CASES])
def test_conv_dense_equals_bucketed(O, dev, delta, T, C_in, C_out):
    """vdt_dvs_conv_dense (bucketing fused into the CuLIF conv, reading the
    spike map) gives conv_bucketed_early's result bit for bit: NCHW and NHWC
    input and output, fan-in up to 1152, T not a multiple of delta (the scan
    runs past T to the end of the last chunk, as the reference's)."""
    from vdttfs import dvs, nets
    spec = nets.dvs_ref(T=T, delta=delta)
    rng = np.random.default_rng(delta * 1000 + C_in)
    N, H, W = 2, 9, 7
    x = spike_map(rng, (N, C_in, H, W), fire=0.35, T=spec.T, edges=True)
    w = (rng.standard_normal((C_out, C_in, 3, 3)) * np.float32(0.35 * np.sqrt(48.0 / C_in))).astype(np.float32)
    off, cin, tin, _ = O.bucketize(x, N * H * W, C_in, spec.T, delta, 0.0, 1, 1, H * W)
    ref = np.empty(N * C_out * H * W, np.float32)
    O.lib().orc_dvs_conv(O._i(off), O._i(cin), O._f(tin), O._f(w), N, C_in, C_out, H, W, 3, spec.T, delta,
                         spec.decay_conv, spec.th_conv, O._f(ref))
    assert 0.0 < np.mean(ref < INF) < 1.0
    wd = dvs.oihw_to_hwio(_t(w, dev))
    assert dvs.dense_supported(C_in, 3)
    got = _np(dvs.conv_dense(_t(x, dev), wd, N, C_in, C_out, H, W, spec))
    assert bits_equal(got, ref), f"{np.sum(got != ref)} of {ref.size} differ"
    xh = np.ascontiguousarray(x.transpose(0, 2, 3, 1))
    got2 = _np(dvs.conv_dense(_t(xh, dev), wd, N, C_in, C_out, H, W, spec, in_layout=0, out_layout=0))
    assert bits_equal(got2.reshape(N, H, W, C_out).transpose(0, 3, 1, 2).reshape(-1), ref)


def test_conv_dense_rejects_large_fan_in(dev):
    from vdttfs import dvs, engine as E, nets
    import torch
    spec = nets.dvs_ref()
    assert not dvs.dense_supported(129, 3)
    x = torch.full((1 * 129 * 4 * 4,), INF, device=dev)
    w = torch.zeros((3, 3, 129, 8), device=dev)
    with pytest.raises(E.VdtError) as ei:
        dvs.conv_dense(x, w, 1, 129, 8, 4, 4, spec)
    assert ei.value.status == 5


def test_run_host_batches_pipelined(dev):
    """dvs.run_host_batches (next batch's frames copied while this batch
    runs) gives each batch run()'s outputs and predictions."""
    import torch
    from vdttfs import dvs, nets, synth
    spec = nets.dvs_ref()
    w = dvs.DvsWeights(spec, synth.dvs_weights(spec, 4), dev)
    frames = [torch.from_numpy(synth.dvs_frames(4, 3, spec, stream=40 + i)).pin_memory() for i in range(3)]
    refs = [dvs.run(spec, w, f.to(dev)) for f in frames]
    outs, preds = dvs.run_host_batches(spec, w, frames)
    for i in range(3):
        assert bits_equal(outs[i].numpy(), _np(refs[i]["out"])), f"batch {i}"
        assert np.array_equal(preds[i].numpy(), _np(refs[i]["pred"]))


@pytest.mark.parametrize("layout", [0, 1])
def test_pool_chunk_early(O, dev, layout):
    from vdttfs import dvs, nets
    spec = nets.dvs_ref()
    rng = np.random.default_rng(3 + layout)
    N, Cc, H, W = 3, 40, 10, 6
    x = spike_map(rng, (N, Cc, H, W), fire=0.5, T=spec.T, edges=True)
    ref = O.dvs_pool(x, N, Cc, H, W, spec)
    xin = x if layout == 1 else x.transpose(0, 2, 3, 1)
    got = _np(dvs.pool(_t(xin, dev), N, Cc, H, W, spec, layout=layout))
    if layout == 0:
        got = got.reshape(N, H // 2, W // 2, Cc).transpose(0, 3, 1, 2).reshape(-1)
    assert bits_equal(got, ref)
    assert np.mean(ref < INF) > 0.05


@pytest.mark.parametrize("th", [0.0, 1.0, 2.5, 5.0])
def test_pool_chunk_early_thresholds(O, dev, th):
    """The pool's scan starts at the chunk of the earliest input spike when
    th > 0 (I and V are exactly 0 before it); th = 0 fires every neuron at
    step 0 through the full scan; sparse inputs leave neurons without any
    spike, T not a multiple of delta makes the scan run past T."""
    import dataclasses
    from vdttfs import dvs, nets
    spec = dataclasses.replace(nets.dvs_ref(T=150, delta=32), th_conv=th)
    rng = np.random.default_rng(int(th * 10) + 7)
    N, Cc, H, W = 2, 24, 10, 8
    x = spike_map(rng, (N, Cc, H, W), fire=0.15, T=spec.T, edges=True)
    ref = O.dvs_pool(x, N, Cc, H, W, spec)
    got = _np(dvs.pool(_t(x, dev), N, Cc, H, W, spec))
    assert bits_equal(got, ref)
    if th == 0.0:
        assert np.all(ref == 0.0)
    else:
        assert 0.0 < np.mean(ref < INF) < 1.0


@pytest.mark.parametrize("F_out", [128, 96, 256])
def test_fc1_recurrent_and_fc2(O, dev, F_out):
    """FC1 (feed-forward sums event-parallel in k_fc1_ff when F_out is a
    multiple of 128, else per neuron inside the recurrent kernel) and FC2
    against the oracle, bit for bit."""
    from vdttfs import dvs, nets, synth
    spec = nets.dvs_ref()
    rng = np.random.default_rng(11 + F_out)
    N, F_in, K = 5, 700, 11
    x = spike_map(rng, (N, F_in), fire=0.3, T=spec.T, edges=True)
    w = (rng.standard_normal((F_out, F_in)) * 0.25).astype(np.float32)
    wr = (rng.standard_normal((F_out, F_out)) * 0.5).astype(np.float32)
    ref1, _ = O.dvs_fc1(x, w, wr, N, F_in, F_out, spec)
    b = dvs.bucketize_rows(_t(x, dev), N, F_in, spec)
    for ws in (True, False):                                 # caller's scratch / library's own
        got1 = _np(dvs.fc1_recurrent(b, _t(w.T, dev), _t(wr.T, dev), N, F_in, F_out, spec, workspace=ws))
        assert bits_equal(got1, ref1), f"workspace={ws}"
    from vdttfs._lib import lib
    need = lib().vdt_dvs_fc1_scratch_bytes(N, F_out, spec.T, spec.delta)
    assert (need > 0) == (F_out % 128 == 0)
    assert 0.0 < np.mean(ref1 < INF) < 1.0
    w2 = (rng.standard_normal((K, F_out)) * 0.8).astype(np.float32)
    ref2, fe, _ = O.dvs_fc2(ref1, w2, N, F_out, K, spec)
    b2 = dvs.bucketize_rows(_t(ref1, dev), N, F_out, spec)
    got2 = _np(dvs.fc2(b2, _t(w2.T, dev), N, F_out, K, spec))
    assert bits_equal(got2, ref2)


@pytest.mark.parametrize("delta", [8, 16, 32])
def test_conv1_raw_early(O, dev, delta):
    from vdttfs import dvs, nets, synth
    spec = nets.dvs_ref(delta=delta)
    spec = nets.DvsSpec(name="t", H=12, W=9, T=spec.T, delta=delta)
    frames = synth.dvs_frames(4, 2, spec, stream=delta)
    w = (np.random.default_rng(delta).standard_normal((spec.convs[0], 2, 3, 3)) * 2.0).astype(np.float32)
    ref = O.dvs_conv1(frames, w, spec, 2)
    got = _np(dvs.conv1_raw(_t(frames, dev), _t(w, dev), spec))
    assert bits_equal(got.reshape(-1), ref)
    assert 0.0 < np.mean(ref < INF) < 1.0


def test_dvs_full_size_network_equals_oracle(O, dev):
    """The 2x128x128 / 11-class configuration of the benchmark, one sample."""
    from vdttfs import dvs, nets, synth
    spec = nets.dvs()
    wts = synth.dvs_weights(spec, 4)
    frames = synth.dvs_frames(4, 1, spec, stream=1)
    ref = O.run_dvs(spec, wts, frames, keep=True)
    r = dvs.run(spec, dvs.DvsWeights(spec, wts, dev), _t(frames, dev), keep=True)
    for i, (a, b) in enumerate(zip(r["maps"], ref["maps"])):
        assert bits_equal(_np(a).reshape(-1), b), f"stage {i} differs"
    assert np.array_equal(_np(r["pred"]), ref["pred"])


# ------------------------------------------- whole network in the C runtime --
def test_dvs_net_c_runtime_matches_the_reference_kernels(dev):
    """The reference's own 2x32x32 network loaded from its flat blob
    (vdt_model_load_dvs_flat) and run by the C++ runtime: the seven stage
    maps of vdt_infer_trace and the graph path's outputs equal the golden
    maps of the reference's kernels, bit for bit."""
    import torch
    from vdttfs import assets, dvs, nets, synth
    g = np.load(os.path.join(GOLDEN, "net_dvs_ref.npz"))
    spec = nets.dvs_ref()
    blob = assets.write_dvs_flat(synth.dvs_weights(spec, 4, gains=DVS_GAINS), spec)
    net = dvs.DvsNet(spec, blob)
    ctx = net.context(4)
    frames = _t(g["frames"].astype(np.float32), dev)
    maps, out, pred = ctx.trace(frames)
    for i, m in enumerate(maps):
        assert bits_equal(_np(m).reshape(-1), g[f"map{i}"].astype(np.float32)), f"stage {DvsNet_stage(i)} differs"
    ref_out = g["map6"].astype(np.float32).reshape(2, spec.classes)
    want = np.array([np.argmin(o) for o in ref_out])
    assert np.array_equal(_np(pred), want)
    o2, p2 = ctx.infer(frames)                                 # captured graph
    assert bits_equal(_np(o2), ref_out) and np.array_equal(_np(p2), want)
    ctx.close()
    net.close()


def DvsNet_stage(i):
    from vdttfs import dvs
    return dvs.DvsNet.STAGES[i]


@pytest.mark.parametrize("graphs", [True, False])
def test_dvs_net_host_paths_equal_device_path(dev, graphs):
    """vdt_infer_host and the pipelined vdt_infer_host_batches on a task-3
    model give vdt_infer's outputs and predictions for every batch, with and
    without CUDA graphs; a smaller batch than the context's maximum works."""
    import torch
    from vdttfs import dvs, nets, synth
    spec = nets.dvs_ref()
    net = dvs.DvsNet(spec, synth.dvs_weights(spec, 4))
    ctx = net.context(5, graphs=graphs)
    frames = [torch.from_numpy(synth.dvs_frames(4, 3, spec, stream=60 + i)).pin_memory() for i in range(3)]
    refs = []
    for f in frames:
        o, p = ctx.infer(f.to(dev))
        refs.append((_np(o), _np(p)))
    for i, f in enumerate(frames):
        o, p = ctx.infer_host(f)
        assert bits_equal(o, refs[i][0]) and np.array_equal(p, refs[i][1]), f"infer_host batch {i}"
    outs, preds = ctx.infer_host_batches(frames)
    for i in range(3):
        assert bits_equal(outs[i], refs[i][0]) and np.array_equal(preds[i], refs[i][1]), f"pipelined batch {i}"
    # the per-stage Python pipeline agrees with the C runtime
    r = dvs.run(spec, dvs.DvsWeights(spec, synth.dvs_weights(spec, 4), dev), frames[0].to(dev))
    assert bits_equal(_np(r["out"]), refs[0][0])
    ctx.close()
    net.close()


def test_dvs_net_profiling_and_unsupported_calls(dev):
    """Profiling times the seven stages; per-layer integrator choice, LUT
    reads and sub-batches are refused on a task-3 model."""
    import torch
    from vdttfs import dvs, engine as E, nets, synth
    spec = nets.dvs_ref()
    net = dvs.DvsNet(spec, synth.dvs_weights(spec, 4))
    ctx = net.context(2)
    ctx.set_profiling(True)
    ctx.layer_times()
    ctx.infer(torch.from_numpy(synth.dvs_frames(4, 2, spec, stream=3)).to(dev))
    bkt, comp, nb = ctx.layer_times()
    assert nb == 1 and (comp > 0).all()
    assert bkt[dvs.DvsNet.STAGES.index("fc1")] > 0 and bkt[dvs.DvsNet.STAGES.index("fc2")] > 0
    ctx.set_profiling(False)
    for call in (lambda: ctx.set_sub_batches(2), lambda: ctx.layer_kernels(), lambda: ctx.set_layer_kernel(0, 1)):
        with pytest.raises(E.VdtError) as ei:
            call()
        assert ei.value.status == 5
    ctx.close()
    net.close()


def test_dvs_net_sizes_capacity_and_long_blob(O, dev):
    """The task-3 model reports its seven stages and classes; a blob longer
    than the network (the reference reads a fixed-size file) loads the same
    weights; batches of 1 and up to the context's maximum run, and a larger
    one is refused before any launch."""
    import ctypes as C
    import torch
    from vdttfs import assets, dvs, engine as E, nets, synth
    from vdttfs._lib import lib
    spec = nets.dvs_ref()
    wts = synth.dvs_weights(spec, 4)
    blob = assets.write_dvs_flat(wts, spec)
    net = dvs.DvsNet(spec, blob + bytes(4 * 3456))           # 1,292,032 floats, as the reference's file
    nl, nc, wb = C.c_int(), C.c_int(), C.c_size_t()
    assert lib().vdt_model_info(net.h, C.byref(nl), C.byref(nc), C.byref(wb)) == 0
    assert (nl.value, nc.value, wb.value) == (7, spec.classes, len(blob))
    ctx = net.context(3)
    frames = synth.dvs_frames(4, 3, spec, stream=70)
    ref = O.run_dvs(spec, wts, frames)
    for B in (1, 3):
        out, pred = ctx.infer(torch.from_numpy(frames[:B]).to(dev))
        assert bits_equal(_np(out), ref["out"][:B]) and np.array_equal(_np(pred), ref["pred"][:B])
    with pytest.raises(E.VdtError) as ei:
        ctx.infer(torch.from_numpy(synth.dvs_frames(4, 4, spec, stream=71)).to(dev))
    assert ei.value.status == 6                               # VDT_ERR_CAPACITY
    ctx.close()
    net.close()
