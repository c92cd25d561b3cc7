"""Expected outputs of bench.py's workloads, for the parity check bench.py
prints beside its timings.

For every bench configuration, the seeded batch rank 0 times (stream 0, the
configuration's batch per GPU at one GPU) is run through the CPU oracle
(oracle/vdt_oracle.c, pinned bit for bit to the reference's own kernels by
tests/golden/*.npz and tests/test_golden.py; the engine is checked against
the reference kernels at these exact batches by tests/test_gpu_bench_configs.py).
For the strong-scaling configuration (LeNet-5 C2: 65,536 images over the
GPUs) also rank 0's batch at 2, 4 and 8 GPUs (65,536 / N images of stream 0),
stored under "<config>@<batch>".  Stored per batch: the predictions and the
SHA-256 of the output values' bytes (float32, [batch, classes]).  CPU only,
about three minutes.

Usage: python tests/golden/make_bench_parity.py [OUT_FILE]
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "vd-ttfs_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, ROOT)

import oracle as O  # noqa: E402
from vdttfs import nets, synth  # noqa: E402

DEFAULT_OUT = os.path.join(HERE, "bench_parity.npz")


def digest(out) -> str:
    return hashlib.sha256(np.ascontiguousarray(out, np.float32).tobytes()).hexdigest()


def expected(config: str, B: int = 0):
    """(outputs [B, classes], predictions [B]) of a bench configuration's
    rank-0 batch (the configuration's batch at one GPU, or B images), from
    the oracle."""
    import bench
    netname, cfg_id, B0, zf, _ = bench.CONFIGS[config]
    B = B or B0
    if netname in ("dvs", "dvs_ref"):
        spec = nets.dvs() if netname == "dvs" else nets.dvs_ref()
        r = O.run_dvs(spec, synth.dvs_weights(spec, cfg_id), synth.dvs_frames(cfg_id, B, spec, stream=0))
    else:
        net = nets.NETS[netname]()
        img = synth.images(cfg_id, B, net.in_h, net.in_w, net.in_c, zf, stream=0)
        r = O.run_net(net, synth.kaiming_layers(net, cfg_id), O.encode_linear(img, net.T))
    return np.ascontiguousarray(r["out"], np.float32), np.asarray(r["pred"], np.int32)


def main():
    out_file = sys.argv[1] if len(sys.argv) > 1 else DEFAULT_OUT
    d = {}
    cases = [(c, 0) for c in ("vgg16", "lenet5_b1024", "lenet5", "dvs", "dvs_ref")]
    cases += [("lenet5", 65536 // n) for n in (2, 4, 8)]
    for config, B in cases:
        key = config if B == 0 else f"{config}@{B}"
        out, pred = expected(config, B)
        d[f"{key}_batch"] = np.int64(pred.size)
        d[f"{key}_out_sha256"] = np.array(digest(out))
        d[f"{key}_pred"] = pred.astype(np.int8)
        print(key, pred.size, digest(out)[:16], np.bincount(pred + 1)[:12].tolist(), flush=True)
    np.savez_compressed(out_file, **d)
    print(out_file, os.path.getsize(out_file))


if __name__ == "__main__":
    main()
