"""Loaders for the reference's asset files, so real weights and datasets drop
in when a user has them (none ship with the reference).

  image sets   dataset_downloaded/{mnist_test10k,cifar10_float}/{i}.bin: one
               float32 image per file (MNIST 28x28, CIFAR-10 HWC 32x32x3), plus
               label_onehot: N x 10 float32 (t1:250-259, t2:298-308)
  DVS frames   cuda_assets/train_data.bin: N x 2 x H x W x T float32,
               train_labels.bin: N x classes int32 one-hot (t3:243-248)
  DVS weights  cuda_assets/dvsgesture_weights.bin: one flat float32 array,
               layers in the order of dvsgesture_weights_meta.txt (conv1,
               conv2, conv3, recurrent FC1, FC1, FC2; t3:237-241)

The TTFS weight blob of tasks 1-2 is read by vdttfs.blob / vdt_model_load_blob.
"""
from __future__ import annotations

import os

import numpy as np

from . import nets


def load_images(directory: str, n: int, shape: tuple) -> np.ndarray:
    """n images {0..n-1}.bin of `shape` float32 each -> [n, *shape] (NHWC for
    CIFAR: shape (32, 32, 3); MNIST: (28, 28, 1))."""
    per = int(np.prod(shape))
    out = np.empty((n, per), np.float32)
    for i in range(n):
        a = np.fromfile(os.path.join(directory, f"{i}.bin"), dtype="<f4", count=per)
        if a.size != per:
            raise ValueError(f"{i}.bin holds {a.size} floats, expected {per}")
        out[i] = a
    return out.reshape((n,) + tuple(shape))


def load_onehot(path: str, n: int, classes: int = 10, dtype="<f4") -> np.ndarray:
    """Class indices from an n x classes one-hot file (float32 for the image
    sets, int32 for DVS): the class whose entry is > 0.5, as the reference
    reads it (t2:394)."""
    a = np.fromfile(path, dtype=dtype, count=n * classes)
    if a.size != n * classes:
        raise ValueError(f"{path}: {a.size} values, expected {n * classes}")
    a = a.reshape(n, classes).astype(np.float64)
    hot = a > 0.5
    if not np.all(hot.sum(axis=1) == 1):
        raise ValueError(f"{path}: rows are not one-hot")
    return np.argmax(hot, axis=1).astype(np.int32)


def load_dvs_frames(path: str, n: int, spec: nets.DvsSpec) -> np.ndarray:
    """[n, C, H, W, T] float32 event frames (time innermost)."""
    shape = (n, spec.in_c, spec.H, spec.W, spec.T)
    a = np.fromfile(path, dtype="<f4", count=int(np.prod(shape)))
    if a.size != int(np.prod(shape)):
        raise ValueError(f"{path}: {a.size} floats, expected {int(np.prod(shape))}")
    return a.reshape(shape)


def dvs_flat_layout(spec: nets.DvsSpec):
    """(name, shape, float offset) of every layer in the flat DVS blob."""
    c1, c2, c3 = spec.convs
    k = spec.k
    fc1_in = spec.stage_shapes()["fc1_in"]
    shapes = [("conv1", (c1, spec.in_c, k, k)), ("conv2", (c2, c1, k, k)), ("conv3", (c3, c2, k, k)),
              ("fc1_rec", (spec.hidden, spec.hidden)), ("fc1", (spec.hidden, fc1_in)),
              ("fc2", (spec.classes, spec.hidden))]
    out, off = [], 0
    for name, shp in shapes:
        out.append((name, shp, off))
        off += int(np.prod(shp))
    return out, off


def load_dvs_flat(src, spec: nets.DvsSpec) -> dict:
    """The flat DVS weight blob (a path or bytes) -> {name: array} in the
    reference's layouts (OIHW convs, [out, in] FC, [hidden, hidden] recurrent),
    the input of vdttfs.dvs.DvsWeights."""
    layout, total = dvs_flat_layout(spec)
    if isinstance(src, (bytes, bytearray, memoryview)):
        a = np.frombuffer(src, dtype="<f4")
    else:
        a = np.fromfile(src, dtype="<f4")
    # the reference reads a fixed-size file and never touches floats past the
    # last listed layer, so a longer file is accepted
    if a.size < total:
        raise ValueError(f"DVS weight blob holds {a.size} floats, the network needs {total}")
    return {name: a[off:off + int(np.prod(shp))].reshape(shp).astype(np.float32)
            for name, shp, off in layout}


def write_dvs_flat(wts: dict, spec: nets.DvsSpec) -> bytes:
    layout, total = dvs_flat_layout(spec)
    buf = np.empty(total, "<f4")
    for name, shp, off in layout:
        w = np.asarray(wts[name], np.float32)
        if w.shape != shp:
            raise ValueError(f"{name}: shape {w.shape}, expected {shp}")
        buf[off:off + w.size] = w.reshape(-1)
    return buf.tobytes()
