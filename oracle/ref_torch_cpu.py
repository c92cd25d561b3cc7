"""Time the reference's CPU paths: for VGG-16 its pure-torch time-driven TTFS
network (task2_vgg16_cifar10/spikingjelly/baseline_torch.py, the same
dynamics as its SpikingJelly script), for the reference LeNet its SpikingJelly
script (task1_lenet_mnist/spikingjelly/baseline_spikingjelly_mnist.py) with a
test-only stand-in for the one SpikingJelly module it imports (SpikingJelly
0.0.0.0.14 is not installed here): layer.Conv2d / layer.Linear with
step_mode="s" are plain synapses, i.e. torch.nn.Conv2d / torch.nn.Linear.
These are the reported CPU baselines beside the vdttfs_cuda and step-by-step
programs.

The reference's own loader (weights_io.load_layers) reads a seeded synthetic
blob written in its format (the same Kaiming weights as bench.py's
workloads) and its network's run_batch runs on seeded synthetic images (the
bench generator, HWC -> CHW as its data_io does), torch on every host core.
These are different discretisations (a full convolution per time step) from
the event-driven path, so only their speed is reported.
Needs the reference tree ($VDT_REFERENCE, else a directory `reference`
beside this repository), so it runs where the reference is checked out, not
on a GPU box; test infrastructure.  Prints one JSON line.

Usage: python oracle/ref_torch_cpu.py [vgg16|lenet_ref] [images]
"""
import json
import os
import platform
import sys
import tempfile
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
REF = os.environ.get("VDT_REFERENCE") or os.path.join(os.path.dirname(ROOT), "reference")
sys.path.insert(0, os.path.join(ROOT, "vd-ttfs_b200"))


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor()


def load_ref_layers(weights_io, blob_name, layers):
    """The reference's own loader on a synthetic blob in its format."""
    from vdttfs import blob
    with tempfile.TemporaryDirectory() as wd:
        os.makedirs(os.path.join(wd, "exported_models"))
        with open(os.path.join(wd, "exported_models", blob_name), "wb") as f:
            f.write(blob.write_blob(layers))
        cwd = os.getcwd()
        os.chdir(wd)
        try:
            return weights_io.load_layers()
        finally:
            os.chdir(cwd)


def spikingjelly_stand_in():
    """sys.modules entries for spikingjelly.activation_based.layer whose
    single-step Conv2d / Linear are torch.nn's (test-only)."""
    import types
    import torch.nn as nn

    def strip(cls):
        class Synapse(cls):
            def __init__(self, *args, step_mode="s", **kw):
                super().__init__(*args, **kw)
        Synapse.__name__ = cls.__name__
        return Synapse
    layer = types.ModuleType("spikingjelly.activation_based.layer")
    layer.Conv2d, layer.Linear = strip(nn.Conv2d), strip(nn.Linear)
    ab = types.ModuleType("spikingjelly.activation_based")
    ab.layer = layer
    sj = types.ModuleType("spikingjelly")
    sj.activation_based = ab
    sys.modules.update({"spikingjelly": sj, "spikingjelly.activation_based": ab,
                        "spikingjelly.activation_based.layer": layer})


def main():
    import numpy as np
    import torch
    from vdttfs import nets, synth
    which = sys.argv[1] if len(sys.argv) > 1 else "vgg16"
    n = int(sys.argv[2]) if len(sys.argv) > 2 else 8
    threads = os.cpu_count()
    torch.set_num_threads(threads)
    if which == "vgg16":
        sys.path.insert(0, os.path.join(REF, "task2_vgg16_cifar10", "spikingjelly"))
        import baseline_torch as bt                               # noqa: E402  (the reference's module)
        import weights_io                                         # noqa: E402
        net = nets.vgg16()
        model = bt.TTFSNet(load_ref_layers(weights_io, "snn_weights_vgg.bin", synth.kaiming_layers(net, 3)), "cpu")
        img = synth.images(3, n, 32, 32, 3, 0.0)                  # NHWC, the bench's images
        impl, steps = "baseline_torch.py, torch CPU", bt.TIME_STEPS
    else:
        sys.path.insert(0, os.path.join(REF, "task1_lenet_mnist", "spikingjelly"))
        spikingjelly_stand_in()
        import baseline_spikingjelly_mnist as bt                  # noqa: E402  (the reference's module)
        import weights_io                                         # noqa: E402
        net = nets.lenet_ref()
        model = bt.SJLeNet(load_ref_layers(weights_io, "snn_weights.bin", synth.kaiming_layers(net, 1)))
        img = synth.images(1, n, 28, 28, 1, 0.8)
        impl, steps = "baseline_spikingjelly_mnist.py with a torch.nn stand-in for SpikingJelly, torch CPU", bt.TW
    x = torch.from_numpy(np.ascontiguousarray(img.transpose(0, 3, 1, 2)))
    t0 = time.perf_counter()
    pred = model.run_batch(x)
    dt = time.perf_counter() - t0
    print(json.dumps({"impl": "reference CPU path (" + impl + ")", "network": which,
                      "images": n, "batch": n, "seconds": round(dt, 3), "images_per_sec": round(n / dt, 3),
                      "threads": threads, "cpu": cpu_model(), "torch": torch.__version__,
                      "time_steps": steps, "pred": [int(p) for p in pred[:8]]}))


if __name__ == "__main__":
    main()
