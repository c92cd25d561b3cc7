"""Weight-blob reader/writer, byte-compatible with the reference's format.

Layout (little-endian), as read by ``load_weights``
(task1_lenet_mnist/vdttfs_cuda/snn_timesorted_earlyexit.cu:185-206,
task2_vgg16_cifar10/vdttfs_cuda/bench_vgg_eventdriven_timesorted_earlyexit.cu:213-234)
and documented in task1_lenet_mnist/spikingjelly/weights_io.py:1-13::

    int32 num_layers
    per layer:
      int32 ndim; int32 shape[ndim]      ndim 4 -> HWIO [kh, kw, cin, cout]
                                         ndim 2 -> [cin, cout]
      float32 kernel[prod(shape)]
      int32 ndim_b; int32 b_size; float32 bias[b_size]
      int32 ndim_tc; int32 tc_size(=1); float32 tc_fire
      int32 ndim_td; int32 td_size(=1); float32 td

The blob is parsed again, in C++, by ``vdt_model_load_blob``; this module is
the Python mirror used to write synthetic blobs and to inspect them.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass

import numpy as np


@dataclass
class BlobLayer:
    kernel: np.ndarray      # float32, HWIO [kh, kw, cin, cout] or [cin, cout]
    bias: np.ndarray        # float32 [cout]
    tc_fire: float
    td: float

    @property
    def is_conv(self) -> bool:
        return self.kernel.ndim == 4

    @property
    def c_in(self) -> int:
        return int(self.kernel.shape[2] if self.is_conv else self.kernel.shape[0])

    @property
    def c_out(self) -> int:
        return int(self.kernel.shape[-1])


def write_blob(layers: list[BlobLayer]) -> bytes:
    out = [struct.pack("<i", len(layers))]
    for l in layers:
        k = np.ascontiguousarray(l.kernel, dtype="<f4")
        out.append(struct.pack("<i", k.ndim))
        out.append(struct.pack(f"<{k.ndim}i", *k.shape))
        out.append(k.tobytes())
        b = np.ascontiguousarray(l.bias, dtype="<f4")
        out.append(struct.pack("<ii", 1, b.size))
        out.append(b.tobytes())
        out.append(struct.pack("<iif", 1, 1, float(l.tc_fire)))
        out.append(struct.pack("<iif", 1, 1, float(l.td)))
    return b"".join(out)


class BlobError(ValueError):
    pass


def read_blob(buf: bytes) -> list[BlobLayer]:
    """Parse a blob; raises BlobError on truncation or malformed shapes."""
    off = 0
    n = len(buf)

    def ri() -> int:
        nonlocal off
        if off + 4 > n:
            raise BlobError(f"truncated blob at byte {off}")
        v = struct.unpack_from("<i", buf, off)[0]
        off += 4
        return v

    def rf(count: int) -> np.ndarray:
        nonlocal off
        if count < 0 or off + 4 * count > n:
            raise BlobError(f"truncated blob: need {4 * count} bytes at {off}")
        a = np.frombuffer(buf, dtype="<f4", count=count, offset=off).astype(np.float32)
        off += 4 * count
        return a

    L = ri()
    if L <= 0 or L > 4096:
        raise BlobError(f"bad layer count {L}")
    layers = []
    for _ in range(L):
        nd = ri()
        if nd not in (2, 4):
            raise BlobError(f"kernel ndim must be 2 or 4, got {nd}")
        shp = [ri() for _ in range(nd)]
        if any(s <= 0 for s in shp):
            raise BlobError(f"bad kernel shape {shp}")
        k = rf(int(np.prod(shp))).reshape(shp)
        ri()
        b = rf(ri())
        ri(); ri()
        tc = float(rf(1)[0])
        ri(); ri()
        td = float(rf(1)[0])
        if b.size != shp[-1]:
            raise BlobError(f"bias size {b.size} != c_out {shp[-1]}")
        layers.append(BlobLayer(k, b, tc, td))
    if off != n:
        raise BlobError(f"trailing bytes: read {off} of {n}")
    return layers
