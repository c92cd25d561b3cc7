"""Generate the golden fixtures from the reference's own vdttfs_cuda kernels.

Runs on a GPU box: loads oracle/_ref/libref_t{1,2,3}.so (the reference's
unmodified task-1/2/3 programs compiled through the oracle/ref_t*.cu
harnesses), feeds them seeded inputs, and stores inputs + reference outputs as
compressed .npz files.  tests/test_golden.py then pins the CPU oracle against
these fixtures without a GPU.

Usage: python tests/golden/make_golden.py OUT_DIR
"""
import os
import sys
import zlib

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "vd-ttfs_b200"))
sys.path.insert(0, os.path.join(ROOT, "tests"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import torch  # noqa: E402

import refbind  # noqa: E402
from helpers import spike_map  # noqa: E402
from vdttfs import nets, synth  # noqa: E402


def T(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def N(t):
    return t.detach().cpu().numpy()


def times_i16(x):
    x = np.asarray(x, np.float32)
    assert np.all(x == np.round(x)) and x.max() <= 9999, "maps must hold integer spike times"
    return x.astype(np.int16)


def crc(a):
    return np.uint32(zlib.crc32(np.ascontiguousarray(a).tobytes()))


def case_weights(task, i, C_in, C_out, K, is_fc):
    """Weights of golden conv case i, regenerated from a fixed seed by the
    test (tests/test_golden.py) instead of being stored."""
    fan = C_in * (1 if is_fc else K * K)
    shp = (C_in, C_out) if is_fc else (K, K, C_in, C_out)
    r = np.random.default_rng(7000 + 100 * task + i)
    return (r.standard_normal(shp, dtype=np.float32)
            * np.float32(np.sqrt(2.0 / fan) * (1.3 if not is_fc else 1.0))).astype(np.float32)


DVS_GAINS = [3.0, 3.0, 3.0, 1.0, 3.0, 3.0]


def gen_task12(task, out):
    R = refbind.RefT12(task)
    tfs, Tw, dl = R.tfs, R.T, R.decay_len
    lut_mode = 1 if task == 2 else 0
    rng = np.random.default_rng(100 + task)
    # --- LUTs for a spread of constants
    consts = np.array([[34.75016403198242, 0.0, 34.75016403198242, 0.0],
                       [17.452274, 0.0, 17.452274, 0.0], [12.5, 3.25, 40.0, -2.0],
                       [5.0, -1.5, 60.0, 7.75], [100.0, 20.0, 3.0, 0.0]], np.float32)
    dec, th = [], []
    for c in consts:
        d, t = R.update_luts(*[float(v) for v in c])
        dec.append(N(d)); th.append(N(t))
    np.savez_compressed(os.path.join(out, f"luts_t{task}.npz"), consts=consts, decay=np.array(dec),
                        th=np.array(th), T=Tw, decay_len=dl)
    # --- bucketize on edge-heavy inputs, several widths
    bk = {}
    for c_in in (1, 3, 12, 64, 100, 512):
        x = spike_map(rng, (257, c_in), fire=0.4, T=80, edges=True)
        off, cin, tin = R.bucketize(T(x), 257, c_in)
        bk[f"x{c_in}"], bk[f"off{c_in}"], bk[f"cin{c_in}"], bk[f"tin{c_in}"] = x, N(off), N(cin), N(tin)
    np.savez_compressed(os.path.join(out, f"bucketize_t{task}.npz"), T=Tw, chunk=R.chunk, tfs=tfs, **bk)
    # --- conv / fc layers through the reference's k_conv_bucketed
    cases = []
    if task == 2:
        cases = [(3, 8, 8, 64, 128, 3, 0), (2, 4, 4, 256, 512, 3, 0), (2, 5, 6, 3, 64, 3, 0),
                 (4, 1, 1, 512, 512, 1, 1), (4, 1, 1, 512, 10, 1, 1)]
    else:
        cases = [(4, 12, 12, 6, 16, 5, 0), (3, 28, 28, 1, 6, 5, 0), (3, 12, 12, 12, 64, 5, 0),
                 (8, 1, 1, 256, 120, 1, 1), (8, 1, 1, 84, 10, 1, 1)]
    cv = {}
    for i, (B, H, W, C_in, C_out, K, is_fc) in enumerate(cases):
        Wt = case_weights(task, i, C_in, C_out, K, is_fc)
        bias = (rng.standard_normal(C_out) * 0.05).astype(np.float32)
        x = spike_map(rng, (B, H, W, C_in), fire=0.35, T=80, edges=(i == 0))
        Ho, Wo = (H, W) if (task == 2 or is_fc) else (H - K + 1, W - K + 1)
        d, t = R.update_luts(34.75, 0.0, 34.75, 0.0)
        n_cols = B if is_fc else B * H * W
        off, cin, tin = R.bucketize(T(x), n_cols, C_in)
        y = R.conv_bucketed(off, cin, tin, T(Wt), T(bias), d, t, 0, B, 1 if is_fc else H,
                            1 if is_fc else W, C_in, Ho, Wo, C_out, K, is_fc)
        cv.update({f"x{i}": x, f"wcrc{i}": crc(Wt), f"b{i}": bias, f"y{i}": N(y),
                   f"shape{i}": np.array([B, H, W, C_in, Ho, Wo, C_out, K, is_fc], np.int32)})
        cv[f"decay{i}"], cv[f"th{i}"] = N(d), N(t)
    np.savez_compressed(os.path.join(out, f"conv_t{task}.npz"), n=len(cases), T=Tw, chunk=R.chunk,
                        tfs=tfs, lut_mode=lut_mode, **cv)
    # --- pooling, encode (log), vmem
    x = spike_map(rng, (3, 8, 8, 16), fire=0.4, edges=True)
    p = R.pooling(T(x), 3, 8, 8, 16)
    px = rng.random(20000).astype(np.float32)
    px[rng.random(px.size) < 0.2] = 0.0
    px[:5] = [0.0, 1e-6, 1e-5, 1.0, 0.5]
    tc = 34.75016403198242 if task == 2 else 17.452274
    enc = R.encode(T(px), tc, 0.0)
    extra = dict(pool_x=x, pool_y=N(p), px=px, enc=N(enc), enc_tc=tc)
    if task == 2:
        xv = spike_map(rng, (9, 512), fire=0.3, T=80, edges=True)
        Wv = rng.standard_normal((512, 10)).astype(np.float32)
        bv = rng.standard_normal(10).astype(np.float32)
        d, _ = R.update_luts(34.75, 0.0, 34.75, 0.0)
        yv = R.layer_vmem(T(xv), T(Wv), T(bv), d, 9, 512, 10)
        extra.update(vmem_x=xv, vmem_w=Wv, vmem_b=bv, vmem_decay=N(d), vmem_y=N(yv))
    np.savez_compressed(os.path.join(out, f"misc_t{task}.npz"), **extra)
    torch.cuda.synchronize()


def layerwise_ref(R, net, layers, spikes):
    """Per-layer maps through the reference's own kernels (and its LUTs)."""
    B = spikes.shape[0]
    x = T(spikes.reshape(-1))
    maps = []
    for li, (l, bl, shp) in enumerate(zip(net.layers, layers, net.shapes())):
        H_in, W_in, C_in, H_out, W_out, C_out = shp
        tc_i, td_i = (net.tc_in, net.td_in) if li == 0 else (layers[li - 1].tc_fire, layers[li - 1].td)
        d, th = R.update_luts(tc_i, td_i, bl.tc_fire, bl.td)
        if l.out == nets.OUT_VMEM:
            y = R.layer_vmem(x, T(bl.kernel), T(bl.bias), d, B, C_in, C_out)
        else:
            fc = l.kind == nets.KIND_FC
            off, cin, tin = R.bucketize(x, B if fc else B * H_in * W_in, C_in)
            y = R.conv_bucketed(off, cin, tin, T(bl.kernel), T(bl.bias), d, th, max(0, int(np.ceil(bl.td))),
                                B, H_in, W_in, C_in, H_out, W_out, C_out, l.k, fc)
        maps.append(N(y))
        if l.pool_after:
            y = R.pooling(y, B, H_out, W_out, C_out)
        x = y
    return maps


def gen_nets(out):
    for name, task, B, cfg_id, zf in (("lenet5", 1, 16, 1, 0.8), ("lenet_ref", 1, 16, 1, 0.8),
                                      ("vgg16", 2, 2, 3, 0.0)):
        R = refbind.RefT12(task)
        net = nets.NETS[name]()
        layers = synth.kaiming_layers(net, cfg_id)
        img = synth.images(cfg_id, B, net.in_h, net.in_w, net.in_c, zf, stream=11)
        if net.encoder == nets.ENC_LOG:
            spikes = N(R.encode(T(img.reshape(-1)), net.tc_in, net.td_in)).reshape(img.shape)
        else:
            # the reference has no linear encoder; the oracle's is exact arithmetic
            spikes = np.where(img < 1e-5, 9999.0, np.floor((np.float32(1) - img) * np.float32(net.T))).astype(np.float32)
        maps = layerwise_ref(R, net, layers, spikes)
        out_ref, pred, _ = R.run_net(net, layers, spikes, reps=1)
        last = maps[-1].reshape(B, -1)
        assert np.array_equal(last.view(np.int32), out_ref.view(np.int32)), "host path != layerwise"
        d = {"img": img, "spikes": spikes, "pred": pred, "out": out_ref}
        for i, m in enumerate(maps):
            if net.layers[i].out == nets.OUT_VMEM:
                d[f"map{i}"] = m
            else:
                d[f"map{i}"] = times_i16(m)
        np.savez_compressed(os.path.join(out, f"net_{name}.npz"), cfg_id=cfg_id, **d)


def gen_task3(out):
    R = refbind.RefT3()
    spec = nets.dvs_ref()
    assert (R.T, R.chunk, R.classes) == (spec.T, spec.delta, spec.classes)
    rng = np.random.default_rng(303)
    Nn = 2
    frames = synth.dvs_frames(4, Nn, spec, density=0.05, stream=3)
    wts = synth.dvs_weights(spec, 4, gains=DVS_GAINS)
    maps = R.run(spec, wts, frames)
    d = {"frames": frames.astype(np.uint8), "decay_conv": R.decay_conv, "decay_fc": R.decay_fc,
         "th_conv": R.th_conv, "th_fc": R.th_fc, "gains": np.array(DVS_GAINS, np.float32)}
    d.update({f"wcrc_{k}": crc(v) for k, v in wts.items()})
    for i, m in enumerate(maps):
        d[f"map{i}"] = times_i16(m)
    # the generic kernels at non-reference shapes
    x = spike_map(rng, (2, 16, 6, 7), fire=0.3, T=160, edges=True)
    off, cin, tin = R.bucketize_conv(T(x), 2, 16, 6, 7)
    d.update(bx=x, boff=N(off), bcin=N(cin), btin=N(tin))
    np.savez_compressed(os.path.join(out, "net_dvs_ref.npz"), **d)


def main():
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py OUT_DIR")
    out = sys.argv[1]
    os.makedirs(out, exist_ok=True)
    for task in (1, 2):
        gen_task12(task, out)
    gen_nets(out)
    gen_task3(out)
    for f in sorted(os.listdir(out)):
        print(f, os.path.getsize(os.path.join(out, f)))


if __name__ == "__main__":
    main()
