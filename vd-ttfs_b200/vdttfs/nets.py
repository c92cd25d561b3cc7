"""Network topology and time configuration of the vdttfs_cuda path.

The reference keeps topology (padding, where pools go, readout kind, encoder
constants) in each program's ``main`` rather than in the weight blob; these
descriptors carry it explicitly and map one-to-one onto the C-ABI's
``vdt_layer_desc`` / ``vdt_time_cfg`` (include/vdttfs.h).

Named networks:

* ``lenet_ref``  -- the reference's LeNet (conv5x5 1->12 valid, pool,
  conv5x5 12->64, pool, FC 1024->10 firing; argmin readout).
  task1_lenet_mnist/vdttfs_cuda/snn_timesorted_earlyexit.cu:293-305.
* ``lenet5``     -- BASELINE config 1/2 (6/16 channels, FC 256->120->84->10)
  with task-1 semantics (no stagger, T-entry decay LUT indexed by tb).
* ``vgg16``      -- BASELINE config 3 / the reference's VGG-16 with task-2
  semantics: same-pad convs, stagger TIME_FIRE_START=40, (T+1)-entry decay LUT
  indexed by clamp((int)t_in, 0, T), membrane readout + argmax
  (task2_vgg16_cifar10/vdttfs_cuda/bench_vgg_eventdriven_timesorted_earlyexit.cu:343-392,
  layer table task2_vgg16_cifar10/spikingjelly/baseline_torch.py:21-38).
* ``dvs``        -- BASELINE config 4, the task-3 CuLIF network generalised to
  2x128x128 input and 11 classes
  (task3_dvsgesture/vdttfs_cuda/snn_inference_timesorted.cu:267-284).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field, replace

import numpy as np

# Enum values shared with include/vdttfs.h
KIND_CONV, KIND_FC = 0, 1
PAD_VALID, PAD_SAME = 0, 1
OUT_FIRE, OUT_VMEM = 0, 1
LUT_BY_TB, LUT_BY_TIN = 0, 1
READ_ARGMIN_FIRST, READ_ARGMIN_LOWEST, READ_ARGMAX = 0, 1, 2
ENC_NONE, ENC_LOG, ENC_LINEAR = 0, 1, 2


@dataclass(frozen=True)
class LayerSpec:
    kind: int            # KIND_CONV / KIND_FC
    c_in: int
    c_out: int
    k: int = 1           # square kernel size (conv)
    pad: int = PAD_SAME  # PAD_VALID / PAD_SAME (pad = k // 2)
    pool_after: bool = False
    out: int = OUT_FIRE  # OUT_FIRE / OUT_VMEM (last layer only)


@dataclass(frozen=True)
class NetSpec:
    name: str
    in_h: int
    in_w: int
    in_c: int
    layers: tuple
    T: int = 80
    delta: int = 16
    tfs: float = 0.0                 # TIME_FIRE_START (inter-layer stagger)
    lut_mode: int = LUT_BY_TB
    decay_len: int = 80              # T (task 1) or T + 1 (task 2)
    readout: int = READ_ARGMIN_FIRST
    tc_in: float = 17.452274
    td_in: float = 0.0
    vth_init: float = 1.0
    inf_time: float = 9999.0
    encoder: int = ENC_LINEAR

    @property
    def n_chunks(self) -> int:
        return (self.T + self.delta - 1) // self.delta

    def shapes(self):
        """Per layer: (H_in, W_in, C_in, H_out, W_out, C_out); FC layers use 1x1."""
        h, w, c = self.in_h, self.in_w, self.in_c
        out = []
        for l in self.layers:
            if l.kind == KIND_CONV:
                if l.c_in != c:
                    raise ValueError(f"{self.name}: conv c_in {l.c_in} != {c}")
                ho, wo = (h, w) if l.pad == PAD_SAME else (h - l.k + 1, w - l.k + 1)
                out.append((h, w, c, ho, wo, l.c_out))
                h, w, c = ho, wo, l.c_out
            else:
                f = h * w * c
                if l.c_in != f:
                    raise ValueError(f"{self.name}: fc c_in {l.c_in} != flattened {f}")
                out.append((1, 1, f, 1, 1, l.c_out))
                h, w, c = 1, 1, l.c_out
            if l.pool_after:
                h, w = h // 2, w // 2
        return out

    @property
    def n_classes(self) -> int:
        """Output values per image: the last layer's map, flattened (an FC
        layer's classes; a conv layer's [H, W, C] after its pool, if any)."""
        _, _, _, ho, wo, co = self.shapes()[-1]
        if self.layers[-1].pool_after:
            ho, wo = ho // 2, wo // 2
        return ho * wo * co

    def with_time(self, T: int | None = None, delta: int | None = None) -> "NetSpec":
        T = self.T if T is None else T
        delta = self.delta if delta is None else delta
        dl = T + 1 if self.lut_mode == LUT_BY_TIN else T
        return replace(self, T=T, delta=delta, decay_len=dl)


def _conv(ci, co, k=3, pad=PAD_SAME, pool=False):
    return LayerSpec(KIND_CONV, ci, co, k, pad, pool)


def _fc(ci, co, out=OUT_FIRE):
    return LayerSpec(KIND_FC, ci, co, 1, PAD_VALID, False, out)


def lenet_ref(T: int = 80, delta: int = 16) -> NetSpec:
    return NetSpec(
        "lenet_ref", 28, 28, 1,
        (_conv(1, 12, 5, PAD_VALID, True), _conv(12, 64, 5, PAD_VALID, True), _fc(1024, 10)),
        T=T, delta=delta, tfs=0.0, lut_mode=LUT_BY_TB, decay_len=T,
        readout=READ_ARGMIN_FIRST, tc_in=17.452274, encoder=ENC_LOG)


def lenet5(T: int = 80, delta: int = 16) -> NetSpec:
    return NetSpec(
        "lenet5", 28, 28, 1,
        (_conv(1, 6, 5, PAD_VALID, True), _conv(6, 16, 5, PAD_VALID, True),
         _fc(256, 120), _fc(120, 84), _fc(84, 10)),
        T=T, delta=delta, tfs=0.0, lut_mode=LUT_BY_TB, decay_len=T,
        readout=READ_ARGMIN_FIRST, tc_in=17.452274, encoder=ENC_LINEAR)


VGG_PLAN = [(3, 64, False), (64, 64, True), (64, 128, False), (128, 128, True),
            (128, 256, False), (256, 256, False), (256, 256, True),
            (256, 512, False), (512, 512, False), (512, 512, True),
            (512, 512, False), (512, 512, False), (512, 512, True)]


def vgg16(T: int = 80, delta: int = 8) -> NetSpec:
    layers = [_conv(ci, co, 3, PAD_SAME, p) for ci, co, p in VGG_PLAN]
    layers += [_fc(512, 512), _fc(512, 512), _fc(512, 10, OUT_VMEM)]
    return NetSpec(
        "vgg16", 32, 32, 3, tuple(layers),
        T=T, delta=delta, tfs=40.0, lut_mode=LUT_BY_TIN, decay_len=T + 1,
        readout=READ_ARGMAX, tc_in=34.75016403198242, encoder=ENC_LINEAR)


# --------------------------------------------------------------------------
# Task 3 (CuLIF) network.  The constants follow
# task3_dvsgesture/vdttfs_cuda/snn_inference_timesorted.cu:24-27; the decays
# are computed like the reference does (double exp of a float, rounded).
# --------------------------------------------------------------------------
DECAY_CONV = float(np.float32(math.exp(float(np.float32(-1.0) / np.float32(5.0)))))
DECAY_FC = float(np.float32(math.exp(float(np.float32(-1.0) / np.float32(60.0)))))
TH_CONV, TH_FC = 5.0, 10.0


@dataclass(frozen=True)
class DvsSpec:
    name: str = "dvs"
    in_c: int = 2
    H: int = 128
    W: int = 128
    T: int = 160
    delta: int = 32
    convs: tuple = (64, 128, 128)     # conv1 (raw frames), conv2, conv3
    pool_after: tuple = (False, True, True)
    k: int = 3
    hidden: int = 128                 # recurrent FC1 width
    classes: int = 11
    decay_conv: float = DECAY_CONV
    th_conv: float = TH_CONV
    decay_fc: float = DECAY_FC
    th_fc: float = TH_FC

    @property
    def n_chunks(self) -> int:
        return (self.T + self.delta - 1) // self.delta

    def stage_shapes(self):
        """(C, H, W) after conv1, conv2, pool1, conv3, pool2; FC1 in-features."""
        h, w = self.H, self.W
        c1, c2, c3 = self.convs
        s = {"conv1": (c1, h, w), "conv2": (c2, h, w)}
        s["pool1"] = (c2, h // 2, w // 2)
        s["conv3"] = (c3, h // 2, w // 2)
        s["pool2"] = (c3, h // 4, w // 4)
        s["fc1_in"] = c3 * (h // 4) * (w // 4)
        return s


def dvs(H: int = 128, W: int = 128, classes: int = 11, T: int = 160, delta: int = 32) -> DvsSpec:
    return DvsSpec(H=H, W=W, classes=classes, T=T, delta=delta)


def dvs_ref(T: int = 160, delta: int = 32) -> DvsSpec:
    """The reference's own DVS shapes: 2x32x32 input, 10 classes."""
    return DvsSpec(name="dvs_ref", H=32, W=32, classes=10, T=T, delta=delta)


NETS = {"lenet_ref": lenet_ref, "lenet5": lenet5, "vgg16": vgg16}
