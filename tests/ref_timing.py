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
    2x32x32 shapes) as its main runs it per batch: frames and weights already
    on the device, the seven stages and four bucketizations, then the output
    copied back (t3:262-296).  Buffers are allocated once, outside the timing."""
    import torch
    R = refbind.RefT3()
    spec = nets.dvs_ref()
    wts = synth.dvs_weights(spec, 4)
    frames = synth.dvs_frames(4, B, spec, stream=0)
    w = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in wts.items()}
    fr = torch.from_numpy(np.ascontiguousarray(frames)).cuda()
    H = spec.H
    nc = (R.T + R.chunk - 1) // R.chunk
    F = 128 * (H // 4) * (H // 4)
    z = lambda *shape, dt=torch.float32: torch.zeros(shape, dtype=dt, device="cuda")
    c1, c2, p1 = z(B, 64, H, H), z(B, 128, H, H), z(B, 128, H // 2, H // 2)
    c3, p2, f1, f2 = z(B, 128, H // 2, H // 2), z(B, 128, H // 4, H // 4), z(B, 128), z(B, spec.classes)
    off_s, cin_s, tin_s = z(B * H * H, nc + 1, dt=torch.int32), z(B * H * H * 128, dt=torch.int32), z(B * H * H * 128)
    off_f, cin_f, tin_f = z(B, nc + 1, dt=torch.int32), z(B * F, dt=torch.int32), z(B * F)
    P = refbind._p
    out = np.empty(B * spec.classes, np.float32)

    def batch():
        R._call("conv1", P(fr), P(c1), P(w["conv1"]), B)
        R._call("bucketize_conv", P(c1), B, 64, H, H, P(cin_s), P(tin_s), P(off_s))
        R._call("conv", P(cin_s), P(tin_s), P(off_s), P(c2), P(w["conv2"]), B, 64, 128, H, H)
        R._call("pool", P(c2), P(p1), B, 128, H, H)
        R._call("bucketize_conv", P(p1), B, 128, H // 2, H // 2, P(cin_s), P(tin_s), P(off_s))
        R._call("conv", P(cin_s), P(tin_s), P(off_s), P(c3), P(w["conv3"]), B, 128, 128, H // 2, H // 2)
        R._call("pool", P(c3), P(p2), B, 128, H // 2, H // 2)
        R._call("bucketize_fc", P(p2), B, F, P(cin_f), P(tin_f), P(off_f))
        R._call("fc1", P(cin_f), P(tin_f), P(off_f), P(f1), P(w["fc1"]), P(w["fc1_rec"]), B, F)
        R._call("bucketize_fc", P(f1), B, 128, P(cin_f), P(tin_f), P(off_f))
        R._call("fc2", P(cin_f), P(tin_f), P(off_f), P(f2), P(w["fc2"]), B, 128, spec.classes)
        out[:] = f2.cpu().numpy().reshape(-1)

    batch()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        batch()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    pred = np.array([int(np.argmin(o)) for o in out.reshape(B, spec.classes)])
    print(json.dumps({"impl": "reference vdttfs_cuda (own kernels)", "workload": "dvs_ref", "batch": B,
                      "reps": reps, "ms_per_batch": round(ms / reps, 3),
                      "samples_per_sec": round(B * reps / (ms / 1e3), 1), "pred_head": pred[:8].tolist()}))


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
