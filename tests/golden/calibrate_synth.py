"""Choose the per-layer Kaiming gains of the synthetic networks (offline).

For each network, layer by layer, bisect the gain g_l on the CPU oracle so
that the fraction of layer-l neurons that fire is close to TARGET (the
benchmark configurations require >= 20%).  Earlier layers keep their chosen
gains.  The printed lists are pasted into vd-ttfs_b200/vdttfs/synth.py GAINS.

Usage: python tests/golden/calibrate_synth.py [lenet5|vgg16|dvs] [n_images]
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "vd-ttfs_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle as O  # noqa: E402
from vdttfs import nets, synth  # noqa: E402

TARGET = 0.30


def _layer_forward(net, layers, li, x, B):
    l, bl = net.layers[li], layers[li]
    H_in, W_in, C_in, H_out, W_out, C_out = net.shapes()[li]
    tc_i, td_i = (net.tc_in, net.td_in) if li == 0 else (layers[li - 1].tc_fire, layers[li - 1].td)
    lut_d, lut_th = O.update_luts(net.T, net.decay_len, tc_i, td_i, bl.tc_fire, bl.td)
    is_fc = l.kind == nets.KIND_FC
    n_cols = B if is_fc else B * H_in * W_in
    off, cin, tin, _ = O.bucketize(x, n_cols, C_in, net.T, net.delta, net.tfs)
    pad = (l.k // 2) if (l.pad == nets.PAD_SAME and not is_fc) else 0
    y, _ = O.conv_bucketed(off, cin, tin, bl.kernel, bl.bias, lut_d, lut_th, 0, B,
                           H_in, W_in, C_in, H_out, W_out, C_out, l.k, pad, is_fc,
                           net.T, net.delta, net.tfs, net.lut_mode)
    return y


def calibrate_net(net, cfg_id, B, zero_frac):
    base = synth.kaiming_layers(net, cfg_id, gains=[1.0] * len(net.layers))
    img = synth.images(cfg_id, B, net.in_h, net.in_w, net.in_c, zero_frac, stream=99)
    x = O.encode_linear(img, net.T).reshape(-1)
    gains = []
    for li, l in enumerate(net.layers):
        if l.out == nets.OUT_VMEM:
            gains.append(1.0)
            break
        lo, hi = 0.05, 64.0
        for _ in range(22):
            g = (lo * hi) ** 0.5
            layers = list(base)
            layers[li] = synth.BlobLayer(base[li].kernel * np.float32(g), base[li].bias,
                                         base[li].tc_fire, base[li].td)
            y = _layer_forward(net, layers, li, x, B)
            frac = float(np.mean(y < 9999.0))
            if frac < TARGET:
                lo = g
            else:
                hi = g
        g = round((lo * hi) ** 0.5, 4)
        gains.append(g)
        base[li] = synth.BlobLayer(base[li].kernel * np.float32(g), base[li].bias,
                                   base[li].tc_fire, base[li].td)
        y = _layer_forward(net, base, li, x, B)
        H_in, W_in, C_in, H_out, W_out, C_out = net.shapes()[li]
        print(f"  layer {li}: gain {g}  fire {np.mean(y < 9999):.3f}", flush=True)
        if l.pool_after:
            y = O.pool_min(y, B, H_out, W_out, C_out)
        x = y
    return gains


def main():
    which = sys.argv[1] if len(sys.argv) > 1 else "lenet5"
    B = int(sys.argv[2]) if len(sys.argv) > 2 else 8
    if which == "lenet5":
        print(calibrate_net(nets.lenet5(), 1, B, 0.8))
    elif which == "vgg16":
        print(calibrate_net(nets.vgg16(), 3, B, 0.0))
    elif which == "lenet_ref":
        print(calibrate_net(nets.lenet_ref(), 1, B, 0.8))


if __name__ == "__main__":
    main()
