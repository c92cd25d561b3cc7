"""CPU: pin the oracle against golden fixtures produced by the reference's
own vdttfs_cuda kernels (tests/golden/make_golden.py, run on a B200 through
oracle/_ref).  Everything is compared bit for bit."""
import os
import sys
import zlib

import numpy as np
import pytest

from conftest import GOLDEN
from helpers import bits_equal, bucket_valid_equal

sys.path.insert(0, GOLDEN)
from make_golden import DVS_GAINS, case_weights  # noqa: E402


def _crc(a):
    return np.uint32(zlib.crc32(np.ascontiguousarray(a).tobytes()))


def _load(name):
    p = os.path.join(GOLDEN, name)
    if not os.path.exists(p):
        pytest.fail(f"golden fixture {name} missing (tests/golden/make_golden.py)")
    return np.load(p)


@pytest.mark.parametrize("task", [1, 2])
def test_luts_equal_reference_update_LUTs(O, task):
    g = _load(f"luts_t{task}.npz")
    for c, d, th in zip(g["consts"], g["decay"], g["th"]):
        rd, rth = O.update_luts(int(g["T"]), int(g["decay_len"]), *[float(v) for v in c])
        assert bits_equal(rd, d) and bits_equal(rth, th)


@pytest.mark.parametrize("task", [1, 2])
def test_bucketize_equals_reference(O, task):
    g = _load(f"bucketize_t{task}.npz")
    for c_in in (1, 3, 12, 64, 100, 512):
        x = g[f"x{c_in}"]
        off, cin, tin, _ = O.bucketize(x, x.shape[0], c_in, int(g["T"]), int(g["chunk"]), float(g["tfs"]), 0)
        bucket_valid_equal(off, cin, tin, g[f"off{c_in}"], g[f"cin{c_in}"], g[f"tin{c_in}"])


@pytest.mark.parametrize("task", [1, 2])
def test_conv_bucketed_equals_reference(O, task):
    g = _load(f"conv_t{task}.npz")
    Tw, chunk, tfs, lm = int(g["T"]), int(g["chunk"]), float(g["tfs"]), int(g["lut_mode"])
    for i in range(int(g["n"])):
        B, H, W, C_in, Ho, Wo, C_out, K, is_fc = [int(v) for v in g[f"shape{i}"]]
        x = g[f"x{i}"]
        Wt = case_weights(task, i, C_in, C_out, K, is_fc)
        assert _crc(Wt) == g[f"wcrc{i}"], "regenerated weights differ from the golden run's"
        n_cols = B if is_fc else B * H * W
        off, cin, tin, _ = O.bucketize(x, n_cols, C_in, Tw, chunk, tfs, 0)
        pad = (K // 2) if (task == 2 and not is_fc) else 0
        y, _ = O.conv_bucketed(off, cin, tin, Wt, g[f"b{i}"], g[f"decay{i}"], g[f"th{i}"], 0, B,
                               1 if is_fc else H, 1 if is_fc else W, C_in, Ho, Wo, C_out, K, pad,
                               is_fc, Tw, chunk, tfs, lm)
        assert bits_equal(y, g[f"y{i}"]), f"case {i}: {np.sum(y != g[f'y{i}'])} differ"
        assert np.mean(g[f"y{i}"] < 9999) > 0.0


@pytest.mark.parametrize("task", [1, 2])
def test_pool_encode_vmem_equal_reference(O, task):
    g = _load(f"misc_t{task}.npz")
    x = g["pool_x"]
    assert bits_equal(O.pool_min(x, *x.shape), g["pool_y"])
    # the reference encodes with CUDA logf; libm logf may round differently only
    # where tc*ln(x) sits on an integer boundary
    enc = O.encode_log(g["px"], float(g["enc_tc"]), 0.0, 80)
    assert np.mean(enc != g["enc"]) < 1e-3
    if task == 2:
        y = O.layer_vmem(g["vmem_x"], g["vmem_w"], g["vmem_b"], g["vmem_decay"], 9, 512, 10, 80, 40.0)
        assert bits_equal(y, g["vmem_y"])


@pytest.mark.parametrize("name", ["lenet5", "lenet_ref", "vgg16"])
def test_networks_equal_reference(O, name):
    from vdttfs import nets, synth
    g = _load(f"net_{name}.npz")
    net = nets.NETS[name]()
    layers = synth.kaiming_layers(net, int(g["cfg_id"]))
    r = O.run_net(net, layers, g["spikes"], keep=True)
    ri = 0
    for li, l in enumerate(net.layers):
        want = g[f"map{li}"].astype(np.float32).reshape(-1)
        assert bits_equal(r["maps"][ri], want), f"layer {li} differs"
        ri += 2 if l.pool_after else 1
    assert bits_equal(r["out"], g["out"])
    assert np.array_equal(r["pred"], g["pred"])


def test_dvs_ref_network_equals_reference(O):
    from vdttfs import nets
    g = _load("net_dvs_ref.npz")
    spec = nets.dvs_ref()
    assert np.float32(spec.decay_conv) == g["decay_conv"] and np.float32(spec.decay_fc) == g["decay_fc"]
    from vdttfs import synth
    wts = synth.dvs_weights(spec, 4, gains=DVS_GAINS)
    for k, v in wts.items():
        assert _crc(v) == g[f"wcrc_{k}"], f"regenerated {k} differs from the golden run's"
    r = O.run_dvs(spec, wts, g["frames"].astype(np.float32), keep=True)
    for i, m in enumerate(r["maps"]):
        assert bits_equal(m, g[f"map{i}"].astype(np.float32).reshape(-1)), f"stage {i} differs"
    x = g["bx"]
    off, cin, tin, _ = O.bucketize(x, 2 * 6 * 7, 16, 160, 32, 0.0, 1, 1, 42)
    bucket_valid_equal(off, cin, tin, g["boff"], g["bcin"], g["btin"])
