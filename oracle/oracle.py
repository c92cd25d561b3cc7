"""ctypes binding of the CPU oracle (oracle/vdt_oracle.c) + whole-network runners.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / `--impl reference` legs of bench.py, never by the product.

The network runners follow the reference programs' host flow:
  * run_net (tasks 1/2): encode -> per layer {update_LUTs(integ = previous
    layer's (tc_fire, td) or (tc_in, td_in) for layer 0, fire = own);
    k_bucketize; k_conv_bucketed | k_layer_vmem; k_pooling} -> readout
    (task1_lenet_mnist/vdttfs_cuda/snn_timesorted_earlyexit.cu:289-315,
     task2_vgg16_cifar10/vdttfs_cuda/bench_vgg_eventdriven_timesorted_earlyexit.cu:341-392).
  * run_dvs (task 3): conv1_raw_early -> bucketize+conv2 -> pool ->
    bucketize+conv3 -> pool -> bucketize_fc+fc1 recurrent -> bucketize_fc+fc2
    -> argmin (task3_dvsgesture/vdttfs_cuda/snn_inference_timesorted.cu:267-296).
"""
from __future__ import annotations

import ctypes as C
import math
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libvdt_oracle.so")
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "vd-ttfs_b200"))
from vdttfs import nets  # noqa: E402

_lib = None
_fp = C.POINTER(C.c_float)
_ip = C.POINTER(C.c_int)


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH) or (
                os.path.getmtime(LIB_PATH) < os.path.getmtime(os.path.join(HERE, "vdt_oracle.c"))):
            build()
        L = C.CDLL(LIB_PATH)
        L.orc_update_luts.argtypes = [C.c_int, C.c_int, C.c_float, C.c_float, C.c_float,
                                      C.c_float, C.c_float, _fp, _fp]
        L.orc_encode_log.argtypes = [_fp, _fp, C.c_long, C.c_float, C.c_float, C.c_int, C.c_float]
        L.orc_encode_linear.argtypes = [_fp, _fp, C.c_long, C.c_int, C.c_float]
        L.orc_bucketize.argtypes = [_fp, C.c_long, C.c_int, C.c_int, C.c_long, C.c_int, C.c_int,
                                    C.c_float, C.c_int, C.c_float, _ip, _ip, _fp]
        L.orc_bucketize.restype = C.c_longlong
        L.orc_conv_bucketed.argtypes = [_ip, _ip, _fp, _fp, _fp, _fp, _fp, C.c_int,
                                        C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                        C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                        C.c_int, C.c_int, C.c_float, C.c_int, C.c_float, _fp]
        L.orc_conv_bucketed.restype = C.c_longlong
        L.orc_layer_vmem.argtypes = [_fp, _fp, _fp, _fp, C.c_int, C.c_int, C.c_int, C.c_int,
                                     C.c_float, C.c_float, _fp]
        L.orc_pool_min.argtypes = [_fp, _fp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float]
        L.orc_readout.argtypes = [_fp, C.c_int, C.c_int, C.c_int, C.c_float, _ip]
        L.orc_dvs_conv1.argtypes = [_fp, _fp] + [C.c_int] * 8 + [C.c_float, C.c_float, _fp]
        L.orc_dvs_conv.argtypes = [_ip, _ip, _fp, _fp] + [C.c_int] * 8 + [C.c_float, C.c_float, _fp]
        L.orc_dvs_conv.restype = C.c_longlong
        L.orc_dvs_pool.argtypes = [_fp, _fp] + [C.c_int] * 6 + [C.c_float, C.c_float]
        L.orc_dvs_fc1_rec.argtypes = [_ip, _ip, _fp, _fp, _fp] + [C.c_int] * 5 + [C.c_float, C.c_float, _fp]
        L.orc_dvs_fc2.argtypes = [_ip, _ip, _fp, _fp] + [C.c_int] * 5 + [C.c_float, C.c_float, _fp]
        L.orc_dvs_fc2.restype = C.c_longlong
        L.orc_set_threads.argtypes = [C.c_int]
        L.orc_set_threads.restype = C.c_int
        L.orc_set_threads(os.cpu_count() or 1)
        _lib = L
    return _lib


def _f(a):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_fp)


def _i(a):
    assert a.dtype == np.int32 and a.flags.c_contiguous
    return a.ctypes.data_as(_ip)


# ----------------------------------------------------------------- kernels --
def update_luts(T, n_decay, tc_integ, td_integ, tc_fire, td_fire, vth=1.0):
    d = np.zeros(n_decay, np.float32)
    th = np.zeros(T, np.float32)
    lib().orc_update_luts(T, n_decay, tc_integ, td_integ, tc_fire, td_fire, vth, _f(d), _f(th))
    return d, th


def encode_log(img, tc, td, T, inf_time=9999.0):
    img = np.ascontiguousarray(img, np.float32)
    out = np.empty_like(img)
    lib().orc_encode_log(_f(img), _f(out), img.size, tc, td, T, inf_time)
    return out


def encode_linear(img, T, inf_time=9999.0):
    img = np.ascontiguousarray(img, np.float32)
    out = np.empty_like(img)
    lib().orc_encode_linear(_f(img), _f(out), img.size, T, inf_time)
    return out


def bucketize(x, n_cols, c_in, T, delta, tfs=0.0, tb_mode=0, layout=0, hw=1, inf_time=9999.0):
    """Returns (off [n_cols, NC+1], cin [n_cols, c_in], tin [n_cols, c_in], total)."""
    x = np.ascontiguousarray(x, np.float32)
    nc = (T + delta - 1) // delta
    off = np.zeros((n_cols, nc + 1), np.int32)
    cin = np.zeros((n_cols, c_in), np.int32)
    tin = np.zeros((n_cols, c_in), np.float32)
    tot = lib().orc_bucketize(_f(x), n_cols, c_in, layout, hw, T, delta, tfs, tb_mode, inf_time,
                              _i(off), _i(cin), _f(tin))
    if tot < 0:
        raise ValueError("bad bucketize parameters")
    return off, cin, tin, int(tot)


def conv_bucketed(off, cin, tin, kernel, bias, lut_decay, lut_th, t_min, B,
                  H_in, W_in, C_in, H_out, W_out, C_out, K, pad, is_fc,
                  T, delta, tfs, lut_mode, inf_time=9999.0):
    out = np.empty(B * H_out * W_out * C_out, np.float32)
    kernel = np.ascontiguousarray(kernel, np.float32)
    fetched = lib().orc_conv_bucketed(
        _i(off), _i(cin), _f(tin), _f(kernel), _f(np.ascontiguousarray(bias, np.float32)),
        _f(lut_decay), _f(lut_th), t_min, B, H_in, W_in, C_in, H_out, W_out, C_out,
        K, K, pad, pad, int(is_fc), T, delta, tfs, lut_mode, inf_time, _f(out))
    return out, int(fetched)


def layer_vmem(x, kernel, bias, lut_decay, B, C_in, C_out, T, tfs, inf_time=9999.0):
    out = np.empty(B * C_out, np.float32)
    lib().orc_layer_vmem(_f(np.ascontiguousarray(x, np.float32)), _f(np.ascontiguousarray(kernel, np.float32)),
                         _f(np.ascontiguousarray(bias, np.float32)), _f(lut_decay),
                         B, C_in, C_out, T, tfs, inf_time, _f(out))
    return out


def pool_min(x, B, H, W, C, inf_time=9999.0):
    out = np.empty(B * (H // 2) * (W // 2) * C, np.float32)
    lib().orc_pool_min(_f(np.ascontiguousarray(x, np.float32)), _f(out), B, H, W, C, inf_time)
    return out


def readout(out, B, K, mode, inf_time=9999.0):
    pred = np.empty(B, np.int32)
    lib().orc_readout(_f(np.ascontiguousarray(out, np.float32)), B, K, mode, inf_time, _i(pred))
    return pred


# ------------------------------------------------------------ networks ------
def t_min_of(td: float) -> int:
    """t_min = max(0, (int)ceilf(td)) (t1:225, t2:252)."""
    t = int(math.ceil(np.float32(td)))
    return max(0, t)


def run_net(net: nets.NetSpec, layers, spikes, keep=False):
    """Whole network on pre-encoded spike times (NHWC [B, H, W, C]).

    Returns dict(out=last layer output [B, classes], pred=[B], maps=[per-layer
    output maps] if keep, fetched=[per layer], events=[per layer])."""
    B = spikes.shape[0]
    x = np.ascontiguousarray(spikes, np.float32).reshape(-1)
    shapes = net.shapes()
    res = {"maps": [], "fetched": [], "events": []}
    for li, (l, bl, shp) in enumerate(zip(net.layers, layers, shapes)):
        H_in, W_in, C_in, H_out, W_out, C_out = shp
        tc_i, td_i = (net.tc_in, net.td_in) if li == 0 else (layers[li - 1].tc_fire, layers[li - 1].td)
        lut_d, lut_th = update_luts(net.T, net.decay_len, tc_i, td_i, bl.tc_fire, bl.td, net.vth_init)
        is_fc = l.kind == nets.KIND_FC
        if l.out == nets.OUT_VMEM:
            y = layer_vmem(x, bl.kernel, bl.bias, lut_d, B, C_in, C_out, net.T, net.tfs, net.inf_time)
            res["fetched"].append(0)
            res["events"].append(0)
        else:
            n_cols = B if is_fc else B * H_in * W_in
            off, cin, tin, tot = bucketize(x, n_cols, C_in, net.T, net.delta, net.tfs, 0, 0, 1, net.inf_time)
            pad = (l.k // 2) if (l.pad == nets.PAD_SAME and not is_fc) else 0
            y, fe = conv_bucketed(off, cin, tin, bl.kernel, bl.bias, lut_d, lut_th, t_min_of(bl.td), B,
                                  H_in, W_in, C_in, H_out, W_out, C_out, l.k, pad, is_fc,
                                  net.T, net.delta, net.tfs, net.lut_mode, net.inf_time)
            res["fetched"].append(fe)
            res["events"].append(tot)
        if keep:
            res["maps"].append(y.copy())
        if l.pool_after:
            y = pool_min(y, B, H_out, W_out, C_out, net.inf_time)
            if keep:
                res["maps"].append(y.copy())
        x = y
    res["out"] = x.reshape(B, net.n_classes)
    res["pred"] = readout(x, B, net.n_classes, net.readout, net.inf_time)
    return res


def dvs_conv1(frames, w, spec, N):
    c1 = spec.convs[0]
    out = np.empty(N * c1 * spec.H * spec.W, np.float32)
    lib().orc_dvs_conv1(_f(np.ascontiguousarray(frames, np.float32)), _f(np.ascontiguousarray(w, np.float32)),
                        N, spec.in_c, c1, spec.H, spec.W, spec.k, spec.T, spec.delta,
                        spec.decay_conv, spec.th_conv, _f(out))
    return out


def dvs_conv(x, w, N, C_in, C_out, H, W, spec):
    off, cin, tin, tot = bucketize(x, N * H * W, C_in, spec.T, spec.delta, 0.0, 1, 1, H * W)
    out = np.empty(N * C_out * H * W, np.float32)
    fe = lib().orc_dvs_conv(_i(off), _i(cin), _f(tin), _f(np.ascontiguousarray(w, np.float32)),
                            N, C_in, C_out, H, W, spec.k, spec.T, spec.delta,
                            spec.decay_conv, spec.th_conv, _f(out))
    return out, int(fe), tot


def dvs_pool(x, N, C, H, W, spec):
    out = np.empty(N * C * (H // 2) * (W // 2), np.float32)
    lib().orc_dvs_pool(_f(np.ascontiguousarray(x, np.float32)), _f(out), N, C, H, W,
                       spec.T, spec.delta, spec.decay_conv, spec.th_conv)
    return out


def dvs_fc1(x, w, w_rec, N, F_in, F_out, spec):
    off, cin, tin, tot = bucketize(x, N, F_in, spec.T, spec.delta, 0.0, 1, 0, 1)
    out = np.empty(N * F_out, np.float32)
    lib().orc_dvs_fc1_rec(_i(off), _i(cin), _f(tin), _f(np.ascontiguousarray(w, np.float32)),
                          _f(np.ascontiguousarray(w_rec, np.float32)), N, F_in, F_out,
                          spec.T, spec.delta, spec.decay_fc, spec.th_fc, _f(out))
    return out, tot


def dvs_fc2(x, w, N, F_in, F_out, spec):
    off, cin, tin, tot = bucketize(x, N, F_in, spec.T, spec.delta, 0.0, 1, 0, 1)
    out = np.empty(N * F_out, np.float32)
    fe = lib().orc_dvs_fc2(_i(off), _i(cin), _f(tin), _f(np.ascontiguousarray(w, np.float32)),
                           N, F_in, F_out, spec.T, spec.delta, spec.decay_fc, spec.th_fc, _f(out))
    return out, int(fe), tot


def run_dvs(spec: nets.DvsSpec, wts: dict, frames, keep=False):
    N = frames.shape[0]
    s = spec.stage_shapes()
    res = {"maps": []}
    c1 = dvs_conv1(frames, wts["conv1"], spec, N)
    c2, _, _ = dvs_conv(c1, wts["conv2"], N, spec.convs[0], spec.convs[1], spec.H, spec.W, spec)
    p1 = dvs_pool(c2, N, spec.convs[1], spec.H, spec.W, spec)
    h2, w2 = spec.H // 2, spec.W // 2
    c3, _, _ = dvs_conv(p1, wts["conv3"], N, spec.convs[1], spec.convs[2], h2, w2, spec)
    p2 = dvs_pool(c3, N, spec.convs[2], h2, w2, spec)
    f1, _ = dvs_fc1(p2, wts["fc1"], wts["fc1_rec"], N, s["fc1_in"], spec.hidden, spec)
    f2, _, _ = dvs_fc2(f1, wts["fc2"], N, spec.hidden, spec.classes, spec)
    if keep:
        res["maps"] = [c1, c2, p1, c3, p2, f1, f2]
    res["out"] = f2.reshape(N, spec.classes)
    res["pred"] = readout(f2, N, spec.classes, nets.READ_ARGMIN_LOWEST)
    return res
