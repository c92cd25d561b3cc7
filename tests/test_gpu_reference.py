"""GPU: the engine against the reference's own kernels (oracle/_ref), fed the
same inputs on the same device.  Bucket offsets/lists bit-exact; first-spike
maps and predictions bit-exact when the engine uses the reference's libm LUTs.
Skipped only when oracle/_ref was not built (no reference tree at build time).
"""
import numpy as np
import pytest

import refbind
from helpers import bits_equal, bucket_valid_equal, spike_map

pytestmark = pytest.mark.gpu


def _t(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _np(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("task", [1, 2])
def test_bucketize_matches_reference_kernel(dev, task):
    if not refbind.available(task):
        pytest.skip("oracle/_ref not built")
    from vdttfs import engine as E
    R = refbind.RefT12(task)
    rng = np.random.default_rng(task)
    for c_in in (1, 3, 16, 64, 512):
        x = spike_map(rng, (999, c_in), fire=0.4, T=80, edges=True)
        roff, rcin, rtin = R.bucketize(_t(x), 999, c_in)
        cfg = E.time_cfg_raw(R.T, R.chunk, R.tfs)
        off, cin, tin = E.bucketize(_t(x), 999, c_in, cfg)
        bucket_valid_equal(_np(off), _np(cin), _np(tin), _np(roff), _np(rcin), _np(rtin))


@pytest.mark.parametrize("name,task,B,cfg_id,zf", [("vgg16", 2, 8, 3, 0.0), ("lenet5", 1, 64, 1, 0.8),
                                                   ("lenet_ref", 1, 64, 1, 0.8)])
def test_network_matches_reference_program(O, dev, name, task, B, cfg_id, zf):
    """The reference's own host path (update_LUTs + launch_* helpers) vs the
    engine with the same LUT source: outputs and predictions bit-identical."""
    if not refbind.available(task):
        pytest.skip("oracle/_ref not built")
    from vdttfs import engine as E, nets, synth
    R = refbind.RefT12(task)
    net = nets.NETS[name]()
    assert (R.T, R.chunk, R.tfs) == (net.T, net.delta, net.tfs)
    layers = synth.kaiming_layers(net, cfg_id)
    img = synth.images(cfg_id, B, net.in_h, net.in_w, net.in_c, zf, stream=9)
    spikes = O.encode_linear(img, net.T)
    r_out, r_pred, _ = R.run_net(net, layers, spikes, reps=1)
    m = E.Model(net, layers, lut_source=E.LUT_HOST_LIBM)
    ctx = E.Context(m, B)
    out, pred = ctx.infer(_t(spikes))
    import torch
    torch.cuda.synchronize()
    assert bits_equal(_np(out), r_out)
    assert np.array_equal(_np(pred), r_pred)
    # the oracle agrees with the reference too
    ref = O.run_net(net, layers, spikes)
    assert bits_equal(ref["out"], r_out)


def test_dvs_generic_kernels_match_reference(O, dev):
    if not refbind.available(3):
        pytest.skip("oracle/_ref not built")
    from vdttfs import nets, synth
    R = refbind.RefT3()
    spec = nets.dvs_ref()
    frames = synth.dvs_frames(4, 2, spec, stream=8)
    wts = synth.dvs_weights(spec, 4, gains=[3.0, 3.0, 3.0, 1.0, 3.0, 3.0])
    ref_maps = R.run(spec, wts, frames)
    orc = O.run_dvs(spec, wts, frames, keep=True)
    for i, (a, b) in enumerate(zip(ref_maps, orc["maps"])):
        assert bits_equal(a, b), f"task-3 stage {i} differs"
