"""Run the reference's step-by-step (time-driven) CUDA programs on this GPU,
the reported baseline named beside vdttfs_cuda.

Each program's own `main` runs unmodified (oracle/_ref/libref_sbs_*.so, built
by `make -C oracle ref`) inside a scratch directory that holds the files it
opens by relative path: the weight blob (seeded Kaiming weights of the
workload's network, vdttfs.blob format = the reference's), 10,000 seeded
synthetic images as per-image .bin files (the same generator and
distribution as bench.py's workload) and a one-hot label file (class i % 10;
the accuracy the program prints is meaningless on synthetic data).  The
throughput is the one the program measures and prints itself (CUDA events
around its time-step loop).  Prints one JSON line.  Test infrastructure, GPU
only.

Usage: python tests/ref_stepbystep.py [vgg16|vgg16_lut|lenet_ref]
"""
import ctypes
import json
import os
import re
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(ROOT, "vd-ttfs_b200"))

from vdttfs import blob, nets, synth  # noqa: E402

# program -> (library, network, config id, zero fraction, blob name, image dir,
# batch the program runs, images it reads)
PROGRAMS = {
    "vgg16": ("libref_sbs_t2.so", "vgg16", 3, 0.0, "snn_weights_vgg.bin", "cifar10_float", 5000, 10000),
    "vgg16_lut": ("libref_sbs_t2_lut.so", "vgg16", 3, 0.0, "snn_weights_vgg.bin", "cifar10_float", 1000, 10000),
    "lenet_ref": ("libref_sbs_t1.so", "lenet_ref", 1, 0.8, "snn_weights.bin", "mnist_test10k", 10000, 10000),
}


def stage(workdir, name):
    lib, net_name, cfg_id, zf, blob_name, img_dir, _, n_img = PROGRAMS[name]
    net = nets.NETS[net_name]()
    os.makedirs(os.path.join(workdir, "exported_models"), exist_ok=True)
    with open(os.path.join(workdir, "exported_models", blob_name), "wb") as f:
        f.write(blob.write_blob(synth.kaiming_layers(net, cfg_id)))
    d = os.path.join(workdir, "dataset_downloaded", img_dir)
    os.makedirs(d, exist_ok=True)
    imgs = synth.images(cfg_id, n_img, net.in_h, net.in_w, net.in_c, zf)
    for i in range(n_img):
        imgs[i].astype("<f4").tofile(os.path.join(d, f"{i}.bin"))
    lab = np.zeros((n_img, 10), "<f4")
    lab[np.arange(n_img), np.arange(n_img) % 10] = 1.0
    lab.tofile(os.path.join(d, "label_onehot"))


def run(name):
    lib_name = PROGRAMS[name][0]
    lib = ctypes.CDLL(os.path.join(ROOT, "oracle", "_ref", lib_name))
    lib.ref_sbs_run.argtypes = [ctypes.c_char_p]
    lib.ref_sbs_run.restype = ctypes.c_int
    with tempfile.TemporaryDirectory() as wd:
        stage(wd, name)
        log = os.path.join(wd, "stdout.txt")
        sys.stdout.flush()
        saved = os.dup(1)
        fd = os.open(log, os.O_WRONLY | os.O_CREAT | os.O_TRUNC)
        os.dup2(fd, 1)
        try:
            rc = lib.ref_sbs_run(wd.encode())
        finally:
            os.dup2(saved, 1)
            os.close(fd)
            os.close(saved)
        text = open(log).read()
    m = re.findall(r"Throughput\s*:\s*([0-9.eE+-]+)", text)
    return rc, (float(m[-1]) if m else None), text


def main():
    name = sys.argv[1] if len(sys.argv) > 1 else "vgg16"
    rc, ips, text = run(name)
    _, net_name, cfg_id, zf, _, _, batch, n_img = PROGRAMS[name]
    print(json.dumps({"impl": "reference stepbystep_cuda", "program": name, "network": net_name,
                      "config_id": cfg_id, "zero_frac": zf, "batch": batch, "images": n_img,
                      "images_per_sec": ips, "rc": rc,
                      "timing": "the program's own CUDA events around its time-step loop",
                      "stdout_tail": text.strip().splitlines()[-6:]}))
    if rc != 0 or ips is None:
        sys.exit(1)


if __name__ == "__main__":
    main()
