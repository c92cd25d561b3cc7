"""Seeded synthetic workloads standing in for MNIST / CIFAR-10 / DVSGesture.

No dataset items are used or reproduced: inputs are random with the shapes,
value ranges and sparsity the benchmark configurations name, and weights are
seeded Kaiming-normal with a per-layer gain.  Seeds are ``0x5D77F5 + config_id``
(numpy PCG64), so every run and every machine regenerates identical tensors.

Config ids: 1 LeNet-5 (B=1024), 2 LeNet-5 (B=65536 sharded), 3 VGG-16,
4 DVS CuLIF, 5 VGG-16 delta/sparsity/T' sweep.
"""
from __future__ import annotations

import numpy as np

from . import nets
from .blob import BlobLayer

SEED_BASE = 0x5D77F5

# Per-layer gains on the Kaiming std sqrt(2 / fan_in).  Chosen layer by layer
# (tests/golden/calibrate_synth.py, bisection on the CPU oracle over 8 images)
# so that roughly 30% of each layer's neurons fire (>= 20% required).
GAINS = {
    "lenet5": [0.1582, 0.3479, 0.6571, 1.0903, 1.0522],
    "vgg16": [0.3318, 1.2826, 0.5129, 1.4551, 0.6443, 1.0594, 1.1088, 0.8631, 1.1408,
              1.1184, 1.0089, 1.6187, 1.4443, 0.721, 1.0337, 1.0],
    "lenet_ref": [0.1634, 0.3961, 0.7404],
    "dvs": None,
}


def seed_for(config_id: int, stream: int = 0) -> int:
    return SEED_BASE + config_id + 1000003 * stream


def images(config_id: int, B: int, H: int, W: int, C: int, zero_frac: float = 0.0,
           stream: int = 0) -> np.ndarray:
    """Pixels uniform in [0, 1) as float32 NHWC; a Bernoulli(zero_frac) mask
    sets pixels to exactly 0 (no spike).  ``stream`` selects an independent
    substream (used for per-rank shards)."""
    rng = np.random.default_rng(seed_for(config_id, stream))
    x = rng.random((B, H, W, C), dtype=np.float32)
    if zero_frac > 0.0:
        m = rng.random((B, H, W, C), dtype=np.float32) < np.float32(zero_frac)
        x[m] = 0.0
    return x


def kaiming_layers(net: nets.NetSpec, config_id: int, gains=None, tc_fire=None,
                   td: float = 0.0) -> list[BlobLayer]:
    """Seeded Kaiming-normal HWIO / [cin, cout] weights, zero bias.
    tc_fire defaults to the network's input encoding constant tc_in and td to
    0 (so t_min = 0); the trained values live in the reference's unshipped
    blobs."""
    rng = np.random.default_rng(seed_for(config_id, 7))
    tc = net.tc_in if tc_fire is None else tc_fire
    if gains is None:
        gains = GAINS.get(net.name) or [1.0] * len(net.layers)
    out = []
    for l, g in zip(net.layers, gains):
        if l.kind == nets.KIND_CONV:
            shape = (l.k, l.k, l.c_in, l.c_out)
            fan_in = l.k * l.k * l.c_in
        else:
            shape = (l.c_in, l.c_out)
            fan_in = l.c_in
        std = np.float32(g * np.sqrt(2.0 / fan_in))
        k = rng.standard_normal(shape, dtype=np.float32) * std
        out.append(BlobLayer(k.astype(np.float32), np.zeros(l.c_out, np.float32),
                             float(tc), float(td)))
    return out


def dvs_frames(config_id: int, N: int, spec: nets.DvsSpec, density: float = 0.05,
               stream: int = 0) -> np.ndarray:
    """Bernoulli(density) events per (polarity, y, x, time-bin) as a dense
    float32 frame tensor [N, C, H, W, T] (time innermost, the reference's
    raw-input layout)."""
    rng = np.random.default_rng(seed_for(config_id, stream))
    shape = (N, spec.in_c, spec.H, spec.W, spec.T)
    return (rng.random(shape, dtype=np.float32) < np.float32(density)).astype(np.float32)


def dvs_weights(spec: nets.DvsSpec, config_id: int, gains=None) -> dict:
    """OIHW conv weights, [out, in] FC weights and the [hidden, hidden]
    recurrent matrix, in the reference's flat-blob order
    (task3_dvsgesture/cuda_assets/dvsgesture_weights_meta.txt)."""
    rng = np.random.default_rng(seed_for(config_id, 7))
    if gains is None:
        gains = GAINS.get("dvs") or [1.0] * 6
    c1, c2, c3 = spec.convs
    k = spec.k
    s = spec.stage_shapes()

    def kn(shape, fan_in, g):
        return (rng.standard_normal(shape, dtype=np.float32)
                * np.float32(g * np.sqrt(2.0 / fan_in))).astype(np.float32)

    return {
        "conv1": kn((c1, spec.in_c, k, k), spec.in_c * k * k, gains[0]),
        "conv2": kn((c2, c1, k, k), c1 * k * k, gains[1]),
        "conv3": kn((c3, c2, k, k), c2 * k * k, gains[2]),
        "fc1_rec": kn((spec.hidden, spec.hidden), spec.hidden, gains[3]),
        "fc1": kn((spec.hidden, s["fc1_in"]), s["fc1_in"], gains[4]),
        "fc2": kn((spec.classes, spec.hidden), spec.hidden, gains[5]),
    }
