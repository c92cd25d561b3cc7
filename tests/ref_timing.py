"""Time the reference's own vdttfs_cuda VGG-16 / LeNet paths on this GPU.

Drives the reference program's host helpers (update_LUTs with its blocking
copies, launch_conv/launch_fc/launch_pool/launch_fc_vmem with their per-launch
device syncs) through oracle/_ref/libref_t{1,2}.so on the same seeded
workload as bench.py: per repetition one batch = H2D copy of the spike times,
the network, D2H copy of the outputs and the host readout.  Prints one JSON
line.  Test infrastructure (reported baseline), GPU only.

Usage: python tests/ref_timing.py [vgg16|lenet5|dvs_ref] [batch] [reps]
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(ROOT, "vd-ttfs_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, HERE)

import refbind  # noqa: E402
from vdttfs import nets, synth  # noqa: E402


def dvs_ref(B, reps):
    """The reference's task-3 kernel sequence (its own kernels, hard-coded
    2x32x32 shapes) on the device, per batch: H2D of the frames, the seven
    stages, D2H of every stage output."""
    import time
    import torch
    R = refbind.RefT3()
    spec = nets.dvs_ref()
    wts = synth.dvs_weights(spec, 4)
    frames = synth.dvs_frames(4, B, spec, stream=0)
    R.run(spec, wts, frames)                                   # warm-up
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(reps):
        maps = R.run(spec, wts, frames)
    dt = (time.perf_counter() - t0) * 1e3
    pred = np.array([int(np.argmin(o)) for o in maps[-1].reshape(B, spec.classes)])
    print(json.dumps({"impl": "reference vdttfs_cuda (own kernels)", "workload": "dvs_ref", "batch": B,
                      "reps": reps, "ms_per_batch": round(dt / reps, 3),
                      "samples_per_sec": round(B * reps / (dt / 1e3), 1), "pred_head": pred[:8].tolist()}))


def main():
    name = sys.argv[1] if len(sys.argv) > 1 else "vgg16"
    B = int(sys.argv[2]) if len(sys.argv) > 2 else 256
    reps = int(sys.argv[3]) if len(sys.argv) > 3 else 10
    if name == "dvs_ref":
        return dvs_ref(B, reps)
    task, cfg_id, zf = (2, 3, 0.0) if name == "vgg16" else (1, 1, 0.8)
    R = refbind.RefT12(task)
    net = nets.NETS[name]()
    layers = synth.kaiming_layers(net, cfg_id)
    img = synth.images(cfg_id, B, net.in_h, net.in_w, net.in_c, zf, stream=0)
    spikes = np.where(img < 1e-5, 9999.0, np.floor((np.float32(1) - img) * np.float32(net.T))).astype(np.float32)
    R.run_net(net, layers, spikes, reps=2)                     # warm-up
    out, pred, ms = R.run_net(net, layers, spikes, reps=reps)
    print(json.dumps({"impl": "reference vdttfs_cuda (own kernels + host helpers)", "workload": name,
                      "batch": B, "reps": reps, "ms_per_batch": round(ms / reps, 3),
                      "images_per_sec": round(B * reps / (ms / 1e3), 1),
                      "pred_head": pred[:8].tolist()}))


if __name__ == "__main__":
    main()
