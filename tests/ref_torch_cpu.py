"""Time the reference's CPU path for VGG-16: its pure-torch time-driven TTFS
network (task2_vgg16_cifar10/spikingjelly/baseline_torch.py, the same
dynamics as its SpikingJelly script, which is not installed here), the
reported CPU baseline beside the vdttfs_cuda and step-by-step programs.

The reference's own loader (weights_io.load_layers) reads a seeded synthetic
blob written in its format (the same Kaiming weights as bench.py's
workload) and its TTFSNet.run_batch runs on seeded synthetic images (the
bench generator, HWC -> CHW as its data_io does), torch on every host core.
It is a different discretisation (680 global time steps, a full convolution
per step) from the event-driven path, so only its speed is reported.
Needs the reference tree (this machine only); test infrastructure.  Prints
one JSON line.

Usage: python tests/ref_torch_cpu.py [images]
"""
import json
import os
import platform
import sys
import tempfile
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
REF_DIR = os.path.join("/root/reference", "task2_vgg16_cifar10", "spikingjelly")
sys.path.insert(0, os.path.join(ROOT, "vd-ttfs_b200"))


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor()


def main():
    import numpy as np
    import torch
    from vdttfs import blob, nets, synth
    n = int(sys.argv[1]) if len(sys.argv) > 1 else 8
    threads = os.cpu_count()
    torch.set_num_threads(threads)
    sys.path.insert(0, REF_DIR)
    import baseline_torch as bt                                   # noqa: E402  (the reference's module)
    import weights_io                                             # noqa: E402
    net = nets.vgg16()
    with tempfile.TemporaryDirectory() as wd:
        os.makedirs(os.path.join(wd, "exported_models"))
        with open(os.path.join(wd, "exported_models", "snn_weights_vgg.bin"), "wb") as f:
            f.write(blob.write_blob(synth.kaiming_layers(net, 3)))
        cwd = os.getcwd()
        os.chdir(wd)
        try:
            layers = weights_io.load_layers()
        finally:
            os.chdir(cwd)
    model = bt.TTFSNet(layers, "cpu")
    img = synth.images(3, n, 32, 32, 3, 0.0)                      # NHWC, the bench's images
    x = torch.from_numpy(np.ascontiguousarray(img.transpose(0, 3, 1, 2)))
    t0 = time.perf_counter()
    pred = model.run_batch(x)
    dt = time.perf_counter() - t0
    print(json.dumps({"impl": "reference CPU path (baseline_torch.py, torch CPU)", "network": "vgg16",
                      "images": n, "batch": n, "seconds": round(dt, 3), "images_per_sec": round(n / dt, 3),
                      "threads": threads, "cpu": cpu_model(), "torch": torch.__version__,
                      "time_steps": bt.TIME_STEPS, "pred": [int(p) for p in pred[:8]]}))


if __name__ == "__main__":
    main()
