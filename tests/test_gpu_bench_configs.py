"""GPU parity at the exact configurations bench.py times.

Kernel choice, grid sizes, the sub-batch split and k_thread's fused pool all
depend on the batch size, so the benchmarked paths are checked here at the
benchmarked sizes, through the same context settings bench.py uses (CUDA
graphs on, each batch as two sub-batches on two streams), against:

* the reference's own vdttfs_cuda kernels and host helpers (oracle/_ref,
  compiled unmodified from the reference sources), bit for bit: VGG-16 C3 at
  B=256 (outputs, predictions and every layer's first-spike map), LeNet-5 C1
  at B=1024 and LeNet-5 C2 at B=65,536 (the whole one-GPU batch, k_thread with
  its pool fused into conv2);
* the CPU oracle (pinned to the reference's kernels by tests/golden) for the
  task-3 network at its full 2x128x128, T=160 shape (DVS C4) on 4 samples.

The engine runs with the reference's host-libm LUTs (bench.py does the same),
so every comparison is bit for bit.  Skipped only when oracle/_ref was not
built (no reference tree at build time).
"""
import numpy as np
import pytest

import refbind
from helpers import bits_equal

pytestmark = pytest.mark.gpu


def _np(t):
    return t.detach().cpu().numpy()


def _bench_case(name, cfg_id, B, zf):
    """The seeded batch bench.py feeds rank 0 (stream 0) and its weights."""
    from vdttfs import nets, synth
    net = nets.NETS[name]()
    layers = synth.kaiming_layers(net, cfg_id)
    img = synth.images(cfg_id, B, net.in_h, net.in_w, net.in_c, zf, stream=0)
    return net, layers, img


def _bench_context(net, layers, B):
    from vdttfs import engine as E
    m = E.Model(net, layers, lut_source=E.LUT_HOST_LIBM)
    ctx = E.Context(m, B)
    ctx.set_sub_batches(2)                   # as bench.py
    return m, ctx


def _engine_infer_twice(ctx, img):
    """Two graph launches of the bench path on pixels (the encoder runs on
    the device, as in bench.py); both must give the same bits."""
    import torch
    x = torch.from_numpy(img).cuda()
    outs = []
    for _ in range(2):
        out, pred = ctx.infer(x, pixels=True)
        torch.cuda.synchronize()
        outs.append((_np(out), _np(pred)))
    assert bits_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][1], outs[1][1]), \
        "two launches of the same graph differ"
    return outs[0]


@pytest.mark.parametrize("name,task,cfg_id,B,zf", [
    ("vgg16", 2, 3, 256, 0.0),        # C3, one GPU
    ("lenet5", 1, 1, 1024, 0.8),      # C1
    ("lenet5", 1, 2, 65536, 0.8),     # C2, the whole batch on one GPU
], ids=["vgg16_C3_B256", "lenet5_C1_B1024", "lenet5_C2_B65536"])
def test_bench_path_matches_reference_program(O, dev, name, task, cfg_id, B, zf):
    """The bench context's output and predictions equal those of the
    reference's own host path (update_LUTs + launch_* helpers, t2:339-398 /
    t1:289-315) on the same batch, bit for bit."""
    if not refbind.available(task):
        pytest.skip("oracle/_ref not built")
    from vdttfs import engine as E
    net, layers, img = _bench_case(name, cfg_id, B, zf)
    R = refbind.RefT12(task)
    assert (R.T, R.chunk, R.tfs) == (net.T, net.delta, net.tfs)
    spikes = O.encode_linear(img, net.T)
    r_out, r_pred, _ = R.run_net(net, layers, spikes, reps=1)
    m, ctx = _bench_context(net, layers, B)
    kinds = ctx.layer_kernels()
    if name == "lenet5":
        assert kinds[:2] == [E.KERNEL_THREAD, E.KERNEL_THREAD], kinds   # conv2 + fused pool
    else:
        assert E.KERNEL_DENSE in kinds and E.KERNEL_SORTED in kinds, kinds
    out, pred = _engine_infer_twice(ctx, img)
    n_bad = int(np.sum(out.view(np.int32) != r_out.view(np.int32)))
    assert n_bad == 0, f"{n_bad} of {out.size} output values differ from the reference program"
    assert np.array_equal(pred, r_pred), f"{int(np.sum(pred != r_pred))} predictions differ"
    # bench.py's end-to-end call: pinned host pixels in, host outputs back,
    # the sub-batches' copies overlapped with each other's compute
    import torch
    h_in = torch.from_numpy(img).pin_memory()
    h_out = torch.empty(out.shape, dtype=torch.float32).pin_memory()
    h_pred = torch.empty(pred.shape, dtype=torch.int32).pin_memory()
    for _ in range(2):
        ctx.infer_host(h_in, pixels=True, out=h_out, pred=h_pred)
        assert bits_equal(h_out.numpy(), r_out) and np.array_equal(h_pred.numpy(), r_pred), "vdt_infer_host"
    fired = np.mean(r_out < net.inf_time) if net.readout != 2 else 1.0
    assert fired > 0.0, "no output neuron fired: the case tests nothing"
    ctx.close()
    m.close()


def test_vgg16_c3_b256_every_layer_map_matches_reference_kernels(O, dev):
    """Every layer's first-spike map at B=256 (the bench batch) against the
    reference's kernels run stage by stage on the same spike times."""
    if not refbind.available(2):
        pytest.skip("oracle/_ref not built")
    import torch
    net, layers, img = _bench_case("vgg16", 3, 256, 0.0)
    R = refbind.RefT12(2)
    spikes = O.encode_linear(img, net.T)
    r_maps, r_out = R.run_layers(net, layers, spikes)
    m, ctx = _bench_context(net, layers, 256)
    maps, out, pred = ctx.trace(torch.from_numpy(spikes).cuda())
    torch.cuda.synchronize()
    for li, (a, b) in enumerate(zip(maps, r_maps)):
        a = _np(a).reshape(-1)
        n_bad = int(np.sum(a.view(np.int32) != b.view(np.int32)))
        assert n_bad == 0, f"layer {li}: {n_bad} of {b.size} first-spike times differ"
        if li < len(maps) - 1:
            frac = float(np.mean(b < net.inf_time))
            assert 0.0 < frac < 1.0, f"layer {li} fired fraction {frac}: the layer tests nothing"
    assert bits_equal(_np(out), r_out)
    ctx.close()
    m.close()


def test_dvs_c4_full_size_matches_oracle(O, dev):
    """Task 3 at BASELINE config 4's shape (2x128x128 frames, T=160, delta=32,
    11 classes) on 4 samples of the bench's seeded frames, through the
    whole-network C entry point: every output and prediction equals the
    oracle's."""
    import torch
    from vdttfs import dvs, nets, synth
    spec = nets.dvs()
    wts = synth.dvs_weights(spec, 4)
    frames = synth.dvs_frames(4, 4, spec, stream=0)
    ref = O.run_dvs(spec, wts, frames)
    net = dvs.DvsNet(spec, wts)
    ctx = net.context(4)
    out, pred = ctx.infer(torch.from_numpy(frames).cuda())
    torch.cuda.synchronize()
    assert bits_equal(_np(out), ref["out"])
    assert np.array_equal(_np(pred), ref["pred"])
    assert np.mean(ref["out"] < 9999.0) > 0.0
    ctx.close()
    net.close()
