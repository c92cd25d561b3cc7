"""ctypes binding of oracle/_ref/libref_*.so: the reference's own
vdttfs_cuda kernels and host helpers, and its step-by-step programs, compiled
unmodified from the reference sources (oracle/ref_t*.cu, oracle/ref_sbs.cu
harnesses).  GPU-only test infrastructure: it pins the CPU oracle and the
engine to the reference itself (tests/), and times the reference as the
reported baselines beside the engine (bench.py's reference legs).  Device
memory comes from torch."""
import ctypes as C
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(ROOT, "oracle", "_ref")
_vp, _i, _f = C.c_void_p, C.c_int, C.c_float


def available(task: int) -> bool:
    return os.path.exists(os.path.join(REF_DIR, f"libref_t{task}.so"))


def _p(t):
    return C.c_void_p(0 if t is None else int(t.data_ptr()))


class RefT12:
    """Tasks 1 and 2 share the kernel signatures."""

    def __init__(self, task: int):
        self.task = task
        L = C.CDLL(os.path.join(REF_DIR, f"libref_t{task}.so"))
        pre = f"ref_t{task}_"
        self.L, self.pre = L, pre
        sig = {
            "info": [C.POINTER(_i), C.POINTER(_i), C.POINTER(_f), C.POINTER(_f), C.POINTER(_f)],
            "update_luts": [_vp, _vp, _f, _f, _f, _f],
            "encode": [_vp, _vp, _i, _f, _f],
            "bucketize": [_vp, _i, _i, _vp, _vp, _vp],
            "conv_bucketed": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i,
                              _i, _i, _i, _i],
            "pooling": [_vp, _vp, _i, _i, _i, _i],
        }
        if task == 2:
            sig["layer_vmem"] = [_vp, _vp, _vp, _vp, _vp, _i, _i, _i]
            sig["run_vgg"] = [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, C.POINTER(_f)]
        else:
            sig["run_net"] = [_i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _f, _f, _vp, _vp, _vp,
                              _i, C.POINTER(_f)]
        for k, a in sig.items():
            f = getattr(L, pre + k)
            f.argtypes = a
            f.restype = C.c_int
        T, ch, tfs, vth, inf = _i(), _i(), _f(), _f(), _f()
        getattr(L, pre + "info")(C.byref(T), C.byref(ch), C.byref(tfs), C.byref(vth), C.byref(inf))
        self.T, self.chunk, self.tfs, self.vth, self.inf = T.value, ch.value, tfs.value, vth.value, inf.value
        self.decay_len = self.T + 1 if task == 2 else self.T

    def _call(self, name, *args):
        st = getattr(self.L, self.pre + name)(*args)
        if st != 0:
            raise RuntimeError(f"{self.pre}{name} failed with CUDA error {st}")

    def update_luts(self, tc_i, td_i, tc_f, td_f):
        import torch
        d = torch.empty(self.decay_len, dtype=torch.float32, device="cuda")
        th = torch.empty(self.T, dtype=torch.float32, device="cuda")
        self._call("update_luts", _p(d), _p(th), tc_i, td_i, tc_f, td_f)
        return d, th

    def encode(self, px, tc, td):
        import torch
        out = torch.empty_like(px)
        self._call("encode", _p(px), _p(out), px.numel(), tc, td)
        return out

    def bucketize(self, x, n_cols, c_in):
        import torch
        nc = (self.T + self.chunk - 1) // self.chunk
        off = torch.zeros((n_cols, nc + 1), dtype=torch.int32, device="cuda")
        cin = torch.zeros((n_cols, c_in), dtype=torch.int32, device="cuda")
        tin = torch.zeros((n_cols, c_in), dtype=torch.float32, device="cuda")
        self._call("bucketize", _p(x), n_cols, c_in, _p(cin), _p(tin), _p(off))
        return off, cin, tin

    def conv_bucketed(self, off, cin, tin, W, bias, d, th, t_min, B, H_in, W_in, C_in, H_out,
                      W_out, C_out, K, is_fc):
        import torch
        out = torch.empty(B * H_out * W_out * C_out, dtype=torch.float32, device="cuda")
        self._call("conv_bucketed", _p(out), _p(cin), _p(tin), _p(off), _p(W), _p(bias), _p(d),
                   _p(th), t_min, B, H_in, W_in, C_in, H_out, W_out, C_out, K, K, int(is_fc))
        return out

    def layer_vmem(self, x, W, bias, d, B, C_in, C_out):
        import torch
        out = torch.empty(B * C_out, dtype=torch.float32, device="cuda")
        self._call("layer_vmem", _p(x), _p(out), _p(W), _p(bias), _p(d), B, C_in, C_out)
        return out

    def pooling(self, x, B, H, W, Cc):
        import torch
        out = torch.empty(B * (H // 2) * (W // 2) * Cc, dtype=torch.float32, device="cuda")
        self._call("pooling", _p(x), _p(out), B, H, W, Cc)
        return out

    def run_layers(self, net, layers, spikes):
        """The reference network stage by stage through the reference's own
        kernels (update_LUTs, k_bucketize, k_conv_bucketed / k_layer_vmem,
        k_pooling), keeping every layer's first-spike map before its pool.
        Returns (maps as flat numpy arrays, last-layer output [B, classes])."""
        import torch
        B = spikes.shape[0]
        x = torch.from_numpy(np.ascontiguousarray(spikes, np.float32)).cuda().reshape(-1)
        maps = []
        for li, (l, bl, shp) in enumerate(zip(net.layers, layers, net.shapes())):
            H_in, W_in, C_in, H_out, W_out, C_out = shp
            tc_i, td_i = (net.tc_in, net.td_in) if li == 0 else (layers[li - 1].tc_fire, layers[li - 1].td)
            d, th = self.update_luts(tc_i, td_i, bl.tc_fire, bl.td)
            W = torch.from_numpy(np.ascontiguousarray(bl.kernel, np.float32)).cuda()
            bias = torch.from_numpy(np.ascontiguousarray(bl.bias, np.float32)).cuda()
            is_fc = l.kind == 1
            if l.out == 1:                                    # membrane readout (task 2 only)
                y = self.layer_vmem(x, W, bias, d, B, C_in, C_out)
            else:
                n_cols = B if is_fc else B * H_in * W_in
                off, cin, tin = self.bucketize(x, n_cols, C_in)
                t_min = max(0, int(np.ceil(np.float32(bl.td))))
                y = self.conv_bucketed(off, cin, tin, W, bias, d, th, t_min, B, H_in, W_in, C_in,
                                       H_out, W_out, C_out, l.k, is_fc)
                del off, cin, tin
            maps.append(y.cpu().numpy())
            if l.pool_after:
                y = self.pooling(y, B, H_out, W_out, C_out)
            x = y
        torch.cuda.synchronize()
        return maps, x.cpu().numpy().reshape(B, -1)

    def run_net(self, net, layers, spikes, reps=1):
        """The reference network through the reference's own host helpers.
        Returns (last-layer output, predictions, milliseconds for `reps`)."""
        import torch
        B = spikes.shape[0]
        dk = [torch.from_numpy(np.ascontiguousarray(l.kernel)).cuda() for l in layers]
        db = [torch.from_numpy(np.ascontiguousarray(l.bias)).cuda() for l in layers]
        kp = (C.c_void_p * len(layers))(*[t.data_ptr() for t in dk])
        bp = (C.c_void_p * len(layers))(*[t.data_ptr() for t in db])
        tc = np.array([l.tc_fire for l in layers], np.float32)
        td = np.array([l.td for l in layers], np.float32)
        x = np.ascontiguousarray(spikes, np.float32)
        K = net.n_classes
        out = np.zeros((B, K), np.float32)
        pred = np.zeros(B, np.int32)
        ms = _f()
        if self.task == 2:
            self._call("run_vgg", B, kp, bp, tc.ctypes.data, td.ctypes.data, x.ctypes.data,
                       out.ctypes.data, pred.ctypes.data, reps, C.byref(ms))
        else:
            shp = []
            for (hi, wi, ci, ho, wo, co), l in zip(net.shapes(), net.layers):
                shp += [hi, wi, ci, ho, wo, co, l.k]
            shp = np.array(shp, np.int32)
            fc = np.array([int(l.kind == 1) for l in net.layers], np.int32)
            pool = np.array([int(l.pool_after) for l in net.layers], np.int32)
            self._call("run_net", B, len(layers), shp.ctypes.data, fc.ctypes.data, pool.ctypes.data,
                       kp, bp, tc.ctypes.data, td.ctypes.data, net.tc_in, net.td_in, x.ctypes.data,
                       out.ctypes.data, pred.ctypes.data, reps, C.byref(ms))
        return out, pred, ms.value


class RefT3:
    def __init__(self):
        L = C.CDLL(os.path.join(REF_DIR, "libref_t3.so"))
        self.L = L
        sig = {
            "info": [C.POINTER(_i)] * 3 + [C.POINTER(_f)] * 4,
            "conv1": [_vp, _vp, _vp, _i],
            "bucketize_conv": [_vp, _i, _i, _i, _i, _vp, _vp, _vp],
            "bucketize_fc": [_vp, _i, _i, _vp, _vp, _vp],
            "conv": [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i],
            "pool": [_vp, _vp, _i, _i, _i, _i],
            "fc1": [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i],
            "fc2": [_vp, _vp, _vp, _vp, _vp, _i, _i, _i],
        }
        for k, a in sig.items():
            f = getattr(L, "ref_t3_" + k)
            f.argtypes = a
            f.restype = C.c_int
        T, ch, ncls = _i(), _i(), _i()
        dc, dfc, thc, thf = _f(), _f(), _f(), _f()
        L.ref_t3_info(C.byref(T), C.byref(ch), C.byref(ncls), C.byref(dc), C.byref(dfc),
                      C.byref(thc), C.byref(thf))
        self.T, self.chunk, self.classes = T.value, ch.value, ncls.value
        self.decay_conv, self.decay_fc, self.th_conv, self.th_fc = dc.value, dfc.value, thc.value, thf.value

    def _call(self, name, *args):
        st = getattr(self.L, "ref_t3_" + name)(*args)
        if st != 0:
            raise RuntimeError(f"ref_t3_{name} failed with CUDA error {st}")

    def _buf(self, *shape, dtype=None):
        import torch
        return torch.zeros(shape, dtype=dtype or torch.float32, device="cuda")

    def bucketize_conv(self, x, N, Cc, H, W):
        import torch
        nc = (self.T + self.chunk - 1) // self.chunk
        off = self._buf(N * H * W, nc + 1, dtype=torch.int32)
        cin = self._buf(N * H * W, Cc, dtype=torch.int32)
        tin = self._buf(N * H * W, Cc)
        self._call("bucketize_conv", _p(x), N, Cc, H, W, _p(cin), _p(tin), _p(off))
        return off, cin, tin

    def bucketize_fc(self, x, N, F):
        import torch
        nc = (self.T + self.chunk - 1) // self.chunk
        off = self._buf(N, nc + 1, dtype=torch.int32)
        cin = self._buf(N, F, dtype=torch.int32)
        tin = self._buf(N, F)
        self._call("bucketize_fc", _p(x), N, F, _p(cin), _p(tin), _p(off))
        return off, cin, tin

    def run(self, spec, wts, frames):
        """The reference's own task-3 kernel sequence (t3:267-284) at its
        hard-coded shapes (2x32x32 input, 64 conv1 channels, 128 hidden)."""
        import torch
        N = frames.shape[0]
        w = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in wts.items()}
        fr = torch.from_numpy(np.ascontiguousarray(frames)).cuda()
        H = spec.H
        c1 = self._buf(N, 64, H, H)
        self._call("conv1", _p(fr), _p(c1), _p(w["conv1"]), N)
        off, cin, tin = self.bucketize_conv(c1, N, 64, H, H)
        c2 = self._buf(N, 128, H, H)
        self._call("conv", _p(cin), _p(tin), _p(off), _p(c2), _p(w["conv2"]), N, 64, 128, H, H)
        p1 = self._buf(N, 128, H // 2, H // 2)
        self._call("pool", _p(c2), _p(p1), N, 128, H, H)
        off, cin, tin = self.bucketize_conv(p1, N, 128, H // 2, H // 2)
        c3 = self._buf(N, 128, H // 2, H // 2)
        self._call("conv", _p(cin), _p(tin), _p(off), _p(c3), _p(w["conv3"]), N, 128, 128, H // 2, H // 2)
        p2 = self._buf(N, 128, H // 4, H // 4)
        self._call("pool", _p(c3), _p(p2), N, 128, H // 2, H // 2)
        F = 128 * (H // 4) * (H // 4)
        off, cin, tin = self.bucketize_fc(p2, N, F)
        f1 = self._buf(N, 128)
        self._call("fc1", _p(cin), _p(tin), _p(off), _p(f1), _p(w["fc1"]), _p(w["fc1_rec"]), N, F)
        off, cin, tin = self.bucketize_fc(f1, N, 128)
        f2 = self._buf(N, spec.classes)
        self._call("fc2", _p(cin), _p(tin), _p(off), _p(f2), _p(w["fc2"]), N, 128, spec.classes)
        torch.cuda.synchronize()
        return [t.cpu().numpy().reshape(-1) for t in (c1, c2, p1, c3, p2, f1, f2)]


# ------------------------------------------ the reference as a reported baseline --
def time_vdttfs_cuda(task, net, layers, spikes, reps=10):
    """The reference's own vdttfs_cuda batch on this GPU, timed the way its
    main times it (t2:337-402 / t1:289-330): per repetition the H2D copy of
    the batch's spike times, every layer through its host helpers (update_LUTs
    with blocking table copies, launch_* with a device sync after each
    launch), the D2H copy of the outputs and the host readout; CUDA events
    around all repetitions.  The spike times come encoded (the synthetic
    workloads' linear encoder, applied on the host), so the timed region
    lacks the reference's one device encode launch.  Returns a dict with the
    milliseconds per batch and the last repetition's outputs / predictions."""
    R = RefT12(task)
    R.run_net(net, layers, spikes, reps=2)                  # warm-up (module load, first launches)
    out, pred, ms = R.run_net(net, layers, spikes, reps=reps)
    return {"ms_per_batch": ms / reps, "out": out, "pred": pred, "reps": reps}


def time_dvs_ref(spec, wts, frames, reps=10):
    """The reference's task-3 kernel sequence (its own kernels at their
    hard-coded 2x32x32 shapes) as its main runs one batch (t3:262-296):
    frames and weights already on the device, the seven stages and four
    bucketizations, the output copied back; buffers allocated once outside
    the timing; CUDA events around all repetitions."""
    import torch
    R = RefT3()
    B = frames.shape[0]
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
    out = np.empty(B * spec.classes, np.float32)

    def batch():
        R._call("conv1", _p(fr), _p(c1), _p(w["conv1"]), B)
        R._call("bucketize_conv", _p(c1), B, 64, H, H, _p(cin_s), _p(tin_s), _p(off_s))
        R._call("conv", _p(cin_s), _p(tin_s), _p(off_s), _p(c2), _p(w["conv2"]), B, 64, 128, H, H)
        R._call("pool", _p(c2), _p(p1), B, 128, H, H)
        R._call("bucketize_conv", _p(p1), B, 128, H // 2, H // 2, _p(cin_s), _p(tin_s), _p(off_s))
        R._call("conv", _p(cin_s), _p(tin_s), _p(off_s), _p(c3), _p(w["conv3"]), B, 128, 128, H // 2, H // 2)
        R._call("pool", _p(c3), _p(p2), B, 128, H // 2, H // 2)
        R._call("bucketize_fc", _p(p2), B, F, _p(cin_f), _p(tin_f), _p(off_f))
        R._call("fc1", _p(cin_f), _p(tin_f), _p(off_f), _p(f1), _p(w["fc1"]), _p(w["fc1_rec"]), B, F)
        R._call("bucketize_fc", _p(f1), B, 128, _p(cin_f), _p(tin_f), _p(off_f))
        R._call("fc2", _p(cin_f), _p(tin_f), _p(off_f), _p(f2), _p(w["fc2"]), B, 128, spec.classes)
        out[:] = f2.cpu().numpy().reshape(-1)

    batch()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        batch()
    e1.record()
    torch.cuda.synchronize()
    o = out.reshape(B, spec.classes)
    return {"ms_per_batch": e0.elapsed_time(e1) / reps, "out": o.copy(),
            "pred": np.array([int(np.argmin(r)) for r in o], np.int32), "reps": reps}


# program -> (library, network, config id, zero fraction, blob name, image dir,
# batch the program runs, images it reads)
STEPBYSTEP = {
    "vgg16": ("libref_sbs_t2.so", "vgg16", 3, 0.0, "snn_weights_vgg.bin", "cifar10_float", 5000, 10000),
    "vgg16_lut": ("libref_sbs_t2_lut.so", "vgg16", 3, 0.0, "snn_weights_vgg.bin", "cifar10_float", 1000, 10000),
    "lenet_ref": ("libref_sbs_t1.so", "lenet_ref", 1, 0.8, "snn_weights.bin", "mnist_test10k", 10000, 10000),
}


def _stage_stepbystep(workdir, name):
    """The files a step-by-step program opens by relative path: the weight
    blob (seeded Kaiming weights of its network, the reference's format),
    seeded synthetic images as per-image .bin files and a one-hot label file
    (class i % 10: the accuracy the program prints means nothing here)."""
    import os
    from vdttfs import blob, nets, synth
    _, net_name, cfg_id, zf, blob_name, img_dir, _, n_img = STEPBYSTEP[name]
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


def run_stepbystep(name):
    """Run one of the reference's step-by-step (time-driven) programs
    unmodified (its own main, oracle/_ref/libref_sbs_*.so) in a scratch
    directory staged by _stage_stepbystep.  Returns a dict with the
    throughput the program measures and prints itself (CUDA events around its
    time-step loop), its return code and the tail of its output."""
    import os
    import re
    import sys
    import tempfile
    lib_name, net_name, cfg_id, zf, _, _, batch, n_img = STEPBYSTEP[name]
    lib = C.CDLL(os.path.join(REF_DIR, lib_name))
    lib.ref_sbs_run.argtypes = [C.c_char_p]
    lib.ref_sbs_run.restype = C.c_int
    with tempfile.TemporaryDirectory() as wd:
        _stage_stepbystep(wd, name)
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
    return {"program": name, "network": net_name, "config_id": cfg_id, "zero_frac": zf, "batch": batch,
            "images": n_img, "images_per_sec": float(m[-1]) if m else None, "rc": rc,
            "timing": "the program's own CUDA events around its time-step loop",
            "stdout_tail": text.strip().splitlines()[-4:]}
