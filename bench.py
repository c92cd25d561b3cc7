"""Benchmark of the B200 VD-TTFS engine (one JSON line on rank 0).

Default workload: BASELINE config 3, the VGG-16 TTFS-SNN at batch 256 per GPU
(T=80, delta=8, TIME_FIRE_START=40), weak scaling over the GPUs of one box.
A step = one batch through the whole network (encode, 15 x {bucketize,
integrate}, 5 pools, membrane readout, argmax) + the NCCL all-gather of the
int32 predictions when N > 1.

  value   images/s over all ranks, input pixels already in HBM, device-timed
          with CUDA events per step (max over ranks); a 256 MiB L2-flush write
          runs between steps, outside the timed events.
  e2e     the same through the host entry points: pinned host pixels -> H2D
          -> the network -> D2H of the logits and predictions, every step
          (vdt_infer_host step by step with the L2 flush between steps; for a
          batch larger than L2, vdt_infer_host_batches, which overlaps step
          i+1's H2D copy with step i's compute).
  roofline  the bucketize + integrator launches of a step (k_bucketize,
          k_dense, k_sorted, k_integrate, k_layer_vmem), timed live with CUDA
          events around each launch (eager profiling pass), against their
          implementation-independent algorithmic bytes (layer_bytes); traffic
          is the DRAM bytes ncu measured for the same launches.
  cpu_baseline  the CPU oracle port (OpenMP over all host cores) on a bounded
          sample of the same workload.

`--impl reference` times the reference algorithm's CPU implementation (the
oracle port; the reference ships no CPU implementation of this path) and
prints its own line; under torchrun only rank 0 works.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "vd-ttfs_b200"))

L2_BYTES = 126 * 1000 * 1000   # B200 L2: a batch larger than this evicts the previous step's data by itself

CONFIGS = {
    # name: (net factory, config id, batch per GPU, zero fraction, scaling)
    "vgg16": ("vgg16", 3, 256, 0.0, "weak"),
    "lenet5": ("lenet5", 2, 65536, 0.8, "strong"),
    "lenet5_b1024": ("lenet5", 1, 1024, 0.8, "weak"),
    "dvs": ("dvs", 4, 64, 0.0, "weak"),     # task-3 CuLIF network, 2x128x128 event frames
    "dvs_ref": ("dvs_ref", 4, 64, 0.0, "weak"),   # the reference's own 2x32x32 DVS network
    "vgg16_sweep": ("vgg16", 5, 256, 0.2, "weak"),   # delta x zero fraction x T'
}

VGG16_DENSE_MACS = 313_725_952      # dense multiply-accumulates of one 3x32x32 VGG-16 image


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="engine", choices=["engine", "reference"])
    ap.add_argument("--config", default="vgg16", choices=sorted(CONFIGS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--batch", type=int, default=0,
                    help="override the config's batch (small cases for profiling; not a bench line)")
    return ap.parse_args()


# ----------------------------------------------------------------- clocks --
class ClockSampler:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index, enabled=True):
        self.gpu = gpu_index
        self.proc = None
        self.enabled = enabled
        self.lines = []

    def start(self):
        if not self.enabled:
            return
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(max(mx)),
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------- peaks --
def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ------------------------------------------------------------- algorithmic --
def layer_bytes(net, events_per_layer, B):
    """Algorithmic bytes of the bucketize + integrate work of each layer for a
    batch of B, implementation-independent: read the input spike map (4 B per
    value), write the first-spike map (4 B per neuron), write and read back
    the bucket lists (8 B per kept event: channel + time) and chunk offsets
    (4 B per column per offset), read the weights once per batch.  The
    membrane-readout layer has no bucket lists."""
    OS = net.n_chunks + 1
    per = []
    for (l, shp, E) in zip(net.layers, net.shapes(), events_per_layer):
        H_in, W_in, C_in, H_out, W_out, C_out = shp
        n_in = B * H_in * W_in * C_in
        n_out = B * H_out * W_out * C_out
        wts = (l.k * l.k if l.kind == 0 else 1) * C_in * C_out
        cols = B if l.kind == 1 else B * H_in * W_in
        lists = 0 if l.out == 1 else 2 * (8 * E + 4 * cols * OS)
        per.append(4 * n_in + 4 * n_out + lists + 4 * wts)
    return per


def launches_per_step(net, kernels, pixels=True):
    """Kernel launches of one inference: encode, per layer bucketize (not for
    k_dense / k_thread / k_layer_vmem layers) + integrator, pools (a k_thread
    layer's pool is fused into it), readout."""
    from vdttfs.engine import KERNEL_DENSE, KERNEL_THREAD, KERNEL_VMEM
    n = 1 if pixels else 0
    for l, k in zip(net.layers, kernels):
        n += 1 if k in (KERNEL_DENSE, KERNEL_THREAD, KERNEL_VMEM) else 2
        n += 1 if l.pool_after and k != KERNEL_THREAD else 0
    return n + 1        # readout


# --------------------------------------------------------------- engine run --
def run_engine(a):
    import torch
    import torch.distributed as dist
    from vdttfs import engine as E, nets, synth

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    netname, cfg_id, Bcfg, zf, scaling = CONFIGS[a.config]
    net = nets.NETS[netname]()
    if a.batch:
        Bcfg = a.batch
    B = Bcfg // world if scaling == "strong" else Bcfg
    layers = synth.kaiming_layers(net, cfg_id)
    img = synth.images(cfg_id, B, net.in_h, net.in_w, net.in_c, zf, stream=rank)
    model = E.Model(net, layers, device=local)
    stream = torch.cuda.Stream(device=dev)
    ctx = E.Context(model, B, stream=stream.cuda_stream)
    ctx.set_sub_batches(2)      # two halves of the batch on two streams (same results)

    x_dev = torch.from_numpy(img).to(dev)
    out = torch.empty((B, net.n_classes), dtype=torch.float32, device=dev)
    pred = torch.empty((B,), dtype=torch.int32, device=dev)
    gathered = torch.empty((world * B,), dtype=torch.int32, device=dev) if world > 1 else None
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def step():
        ctx.infer(x_dev, pixels=True, out=out, pred=pred)
        if world > 1:
            with torch.cuda.stream(stream):
                dist.all_gather_into_tensor(gathered, pred)

    # ---- counters (events / fetched synapses) on one untimed batch
    ctx.set_counting(True)
    with torch.cuda.stream(stream):
        ctx.infer(x_dev, pixels=True, out=out, pred=pred)
    stream.synchronize()
    ev_total, fetched = ctx.counters()
    ctx.set_counting(False)

    # ---- timed device steps
    for _ in range(a.warmup):
        with torch.cuda.stream(stream):
            step()
    stream.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local, enabled=(rank == 0 and not a.no_clocks))
    clocks.start()
    times = []
    for _ in range(a.steps):
        with torch.cuda.stream(stream):
            flush.fill_(1)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            step()
            e1.record(stream)
        stream.synchronize()
        times.append(e0.elapsed_time(e1))
    clk = clocks.stop()
    tot_ms = float(np.sum(times))
    if world > 1:
        t = torch.tensor([tot_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        tot_ms = float(t.item())
    value = world * B * a.steps / (tot_ms / 1e3)

    # ---- end to end through host buffers (pinned), every step.  A batch
    # larger than L2 goes through the pipelined serving call
    # (vdt_infer_host_batches: step i+1's H2D copy overlaps step i's compute,
    # every step's copies inside the timed region); a smaller one step by
    # step with the L2 flush between steps (vdt_infer_host).
    h_in = torch.from_numpy(img).pin_memory()
    pipelined = img.nbytes > L2_BYTES
    if pipelined:
        h_outs = [torch.empty((B, net.n_classes), dtype=torch.float32).pin_memory() for _ in range(max(a.steps, 2))]
        h_preds = [torch.empty((B,), dtype=torch.int32).pin_memory() for _ in range(max(a.steps, 2))]
        ctx.infer_host_batches([h_in] * 2, pixels=True, outs=h_outs[:2], preds=h_preds[:2])   # both slots' graphs
        if world > 1:
            dist.barrier()
        with torch.cuda.stream(stream):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        ctx.infer_host_batches([h_in] * a.steps, pixels=True, outs=h_outs[:a.steps], preds=h_preds[:a.steps])
        with torch.cuda.stream(stream):
            e1.record(stream)
        stream.synchronize()
        e_times = [e0.elapsed_time(e1)]
    else:
        h_out = torch.empty((B, net.n_classes), dtype=torch.float32).pin_memory()
        h_pred = torch.empty((B,), dtype=torch.int32).pin_memory()
        for _ in range(max(1, a.warmup)):
            ctx.infer_host(h_in, pixels=True, out=h_out, pred=h_pred)
        if world > 1:
            dist.barrier()
        e_times = []
        for _ in range(a.steps):
            with torch.cuda.stream(stream):
                flush.fill_(1)
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
            ctx.infer_host(h_in, pixels=True, out=h_out, pred=h_pred)
            with torch.cuda.stream(stream):
                e1.record(stream)
            stream.synchronize()
            e_times.append(e0.elapsed_time(e1))
    e_ms = float(np.sum(e_times))
    if world > 1:
        t = torch.tensor([e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
    e2e = world * B * a.steps / (e_ms / 1e3)

    # ---- integrator roofline: per-launch CUDA events (eager profiling pass)
    ctx.set_profiling(True)
    ctx.layer_times()
    prof_steps = max(3, min(a.steps, 10))
    for _ in range(prof_steps):
        with torch.cuda.stream(stream):
            flush.fill_(1)
            ctx.infer(x_dev, pixels=True, out=out, pred=pred)
    bkt_ms, int_ms, pool_ms, nb = ctx.layer_times()
    ctx.set_profiling(False)
    kernels = ctx.layer_kernels()
    # kept events per layer, from the engine's own bucket offsets
    per_layer_events = layer_events(E, net, layers, x_dev, B, dev)
    lbytes = layer_bytes(net, per_layer_events, B)
    alg_bytes = int(sum(lbytes))
    work_ms = (float(np.sum(bkt_ms)) + float(np.sum(int_ms))) / nb
    peak, peak_kind = peaks()
    achieved = alg_bytes / (work_ms / 1e3) / 1e9

    if world > 1:
        dist.barrier()
    res = None
    if rank == 0:
        res = {
            "metric": "images_per_sec", "value": round(value, 1), "unit": "images/s",
            "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": round(tot_ms / a.steps, 4), "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic (seeded uniform pixels, Kaiming weights, see vdttfs/synth.py)",
            "config": {"workload": f"{netname} C{cfg_id}", "model": netname, "global_batch": world * B,
                       "batch_per_gpu": B, "T": net.T, "delta": net.delta, "fire_start": net.tfs,
                       "zero_frac": zf, "parallelism": f"dp{world}", "l2": "flushed (256 MiB write) between steps",
                       "sub_batches": 2},
            "e2e": {"value": round(e2e, 1), "unit": "images/s",
                    "h2d_bytes_per_step": int(img.nbytes),
                    "d2h_bytes_per_step": int(B * net.n_classes * 4 + B * 4),
                    "api": "vdt_infer_host_batches (pipelined, batch > L2)" if pipelined
                    else "vdt_infer_host per step, L2 flushed between steps"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": traffic_per_step(netname, B),
                         "kernel": "bucketize + integrators, all launches of one step ("
                                   + ", ".join(f"L{i}:{E.KERNEL_NAMES[k]}" for i, k in enumerate(kernels)) + ")",
                         "peak_source": f"{peak_kind} hbm_gbs",
                         "algorithmic_bytes_per_step": alg_bytes,
                         "algorithmic_bytes_per_layer": [int(v) for v in lbytes],
                         "kernel_ms_per_step": round(work_ms, 4),
                         "integrate_ms_per_layer": [round(float(v) / nb, 4) for v in int_ms],
                         "bucketize_ms_per_step": round(float(np.sum(bkt_ms)) / nb, 4),
                         "pool_ms_per_step": round(float(np.sum(pool_ms)) / nb, 4)},
            "gpu_launches": launches_per_step(net, kernels) * a.steps,
            "events_per_image": round(ev_total / B, 1),
            "fetched_synapses_per_image": round(fetched / B, 1),
            "clocks": clk,
        }
        if not a.no_cpu_baseline:
            res["cpu_baseline"] = cpu_baseline(net, layers, img, cfg_id, budget_s=20.0)
    if world > 1:
        del ctx
        dist.destroy_process_group()
    return res


# DRAM bytes (read + write) per image of the bucketize + integrator launches,
# from ncu's dram__bytes_read.sum + dram__bytes_write.sum over one step
# (summary and command in profiles/traffic_vgg16_b256.md).
DRAM_BYTES_PER_IMAGE = {"vgg16": 1310419}


def traffic_per_step(netname, B):
    v = DRAM_BYTES_PER_IMAGE.get(netname)
    return None if v is None else int(round(v * B))


def layer_events(E, net, layers, x_dev, B, dev):
    """Per-layer kept-event counts (exact), from the engine's own counters."""
    from vdttfs import nets
    import torch
    per = []
    # run the network layer by layer through the per-stage API
    maps = None
    ctx = E.Context(E.Model(net, layers, device=dev.index), B)
    maps, _, _ = ctx.trace(x_dev, pixels=True)
    cfg = E.time_cfg(net)
    enc = E.encode_image(x_dev.reshape(-1), net.encoder, net.tc_in, net.td_in, net.T).reshape(x_dev.shape)
    x = enc
    for li, (l, shp) in enumerate(zip(net.layers, net.shapes())):
        H_in, W_in, C_in, H_out, W_out, C_out = shp
        if l.out == nets.OUT_VMEM:
            per.append(0)
        else:
            n_cols = B if l.kind == nets.KIND_FC else B * H_in * W_in
            off, _, _ = E.bucketize(x.reshape(-1), n_cols, C_in, cfg)
            per.append(int(off[:, -1].sum().item()))
        y = maps[li]
        if l.pool_after:
            y = E.pooling(y.reshape(-1), B, H_out, W_out, C_out)
        x = y
    torch.cuda.synchronize()
    ctx.close()
    return per


# --------------------------------------------------------------- CPU legs --
def cpu_baseline(net, layers, img, cfg_id, budget_s=20.0):
    """Oracle port on a bounded sample: grow the sample until one pass takes
    ~budget_s / 4, then time passes until ~budget_s elapsed."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    cores = os.cpu_count() or 1
    n = 2
    while True:
        x = O.encode_linear(img[:n], net.T)
        t0 = time.perf_counter()
        O.run_net(net, layers, x)
        dt = time.perf_counter() - t0
        if dt > budget_s / 4 or n >= img.shape[0]:
            break
        n = min(img.shape[0], n * 2)
    reps, t_tot = 0, 0.0
    while t_tot < budget_s * 0.75 and reps < 8:
        x = O.encode_linear(img[:n], net.T)
        t0 = time.perf_counter()
        O.run_net(net, layers, x)
        t_tot += time.perf_counter() - t0
        reps += 1
    return {"value": round(n * reps / t_tot, 2), "unit": "images/s", "cores": cores, "kind": "port",
            "sample": f"{reps} passes of {n} images of the same workload (linear encode + network), "
                      f"OpenMP over {cores} threads"}


def run_reference(a):
    from vdttfs import nets, synth
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    netname, cfg_id, Bcfg, zf, scaling = CONFIGS[a.config]
    net = nets.NETS[netname]()
    layers = synth.kaiming_layers(net, cfg_id)
    cores = os.cpu_count() or 1
    n = 8 if netname == "vgg16" else 512
    img = synth.images(cfg_id, n, net.in_h, net.in_w, net.in_c, zf, stream=0)
    for _ in range(a.warmup):
        O.run_net(net, layers, O.encode_linear(img, net.T))
    t0 = time.perf_counter()
    for _ in range(a.steps):
        O.run_net(net, layers, O.encode_linear(img, net.T))
    dt = time.perf_counter() - t0
    v = round(n * a.steps / dt, 2)
    return {"impl": "reference", "metric": "images_per_sec", "value": v, "unit": "images/s",
            "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": round(dt / a.steps * 1e3, 3), "higher_is_better": True, "scaling": scaling,
            "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
            "config": {"workload": f"{netname} C{cfg_id}", "model": netname, "batch_per_step": n,
                       "T": net.T, "delta": net.delta},
            "cpu_baseline": {"value": v, "unit": "images/s", "cores": cores, "kind": "port",
                             "sample": f"{n} images per step, the CPU port of the reference's "
                                       f"vdttfs algorithm (oracle/vdt_oracle.c), OpenMP {cores} threads"},
            "e2e": {"value": v, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ------------------------------------------------------------ DVS (task 3) --
def dvs_stages(dvs, spec, w, x, N, marks=None):
    """The DVS pipeline stage by stage; with `marks`, a CUDA event pair
    brackets every stage.  Returns (outputs, predictions, event counts)."""
    import torch
    s = spec.stage_shapes()
    c1n, c2n, c3n = spec.convs
    H, W, H2, W2 = spec.H, spec.W, spec.H // 2, spec.W // 2
    ev = {}

    def mark(name, fn):
        if marks is None:
            return fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        r = fn()
        e1.record()
        marks.append((name, e0, e1))
        return r

    spec0, spec = spec, dvs.internal_spec(spec)
    def conv(name, y, wt, cin, cout, h, wd):
        # the fused kernel (bucketing inside the conv) where it applies, as dvs.run
        if dvs.dense_supported(cin, spec.k):
            ev[name] = None
            return mark(name, lambda: dvs.conv_dense(y, wt, N, cin, cout, h, wd, spec))
        b = mark("bucketize", lambda: dvs.bucketize_sites(y, N, cin, h, wd, spec))
        ev[name] = b
        return mark(name, lambda: dvs.conv_bucketed(b, wt, N, cin, cout, h, wd, spec))

    y = mark("conv1_raw", lambda: dvs.conv1_raw(x, w.conv1, spec0))
    y = conv("conv2", y, w.conv2, c1n, c2n, H, W)
    y = mark("pool1", lambda: dvs.pool(y, N, c2n, H, W, spec))
    y = conv("conv3", y, w.conv3, c2n, c3n, H2, W2)
    y = mark("pool2", lambda: dvs.pool(y, N, c3n, H2, W2, spec))
    b = mark("bucketize", lambda: dvs.bucketize_rows(y, N, s["fc1_in"], spec))
    ev["fc1"] = b
    y = mark("fc1", lambda: dvs.fc1_recurrent(b, w.fc1_t, w.rec_t, N, s["fc1_in"], spec.hidden, spec))
    b = mark("bucketize", lambda: dvs.bucketize_rows(y, N, spec.hidden, spec))
    ev["fc2"] = b
    y = mark("fc2", lambda: dvs.fc2(b, w.fc2_t, N, spec.hidden, spec.classes, spec))
    from vdttfs import engine as E, nets
    pred = mark("readout", lambda: E.readout(y, N, spec.classes, nets.READ_ARGMIN_LOWEST))
    return y, pred, ev


def dvs_bytes(spec, N, ev):
    """Algorithmic bytes of one DVS batch: every stage's input map read and
    output map written once (conv1: the dense frames), the bucketed stages'
    lists written and read back (8 B per kept event, 4 B per chunk offset;
    none for a conv that reads its input map itself), the weights once."""
    s = spec.stage_shapes()
    c1n, c2n, c3n = spec.convs
    HW, HW2, HW4 = spec.H * spec.W, spec.H * spec.W // 4, spec.H * spec.W // 16
    OS = spec.n_chunks + 1
    k2 = spec.k * spec.k
    # a fused conv (ev[name] None) writes and reads no lists
    lists = lambda name, cols: 0 if ev[name] is None else 2 * (8 * int(ev[name][0][:, -1].sum().item()) + 4 * cols * OS)
    b = 4 * N * spec.in_c * HW * spec.T + 4 * N * c1n * HW + 4 * c1n * spec.in_c * k2          # conv1
    b += 4 * N * c1n * HW + 4 * N * c2n * HW + lists("conv2", N * HW) + 4 * c2n * c1n * k2    # conv2
    b += 4 * N * c2n * HW + 4 * N * c2n * HW2                                                    # pool1
    b += 4 * N * c2n * HW2 + 4 * N * c3n * HW2 + lists("conv3", N * HW2) + 4 * c3n * c2n * k2  # conv3
    b += 4 * N * c3n * HW2 + 4 * N * c3n * HW4                                                   # pool2
    b += 4 * N * s["fc1_in"] + 4 * N * spec.hidden + lists("fc1", N) + 4 * s["fc1_in"] * spec.hidden \
        + 4 * spec.hidden * spec.hidden                                                         # fc1
    b += 4 * N * spec.hidden + 4 * N * spec.classes + lists("fc2", N) + 4 * spec.hidden * spec.classes
    return b


def run_dvs_engine(a):
    import torch
    import torch.distributed as dist
    from vdttfs import dvs, nets, synth

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    netname, cfg_id, Bcfg, _, scaling = CONFIGS[a.config]
    B = a.batch or Bcfg
    spec = nets.dvs() if netname == "dvs" else nets.dvs_ref()
    wts = synth.dvs_weights(spec, cfg_id)
    w = dvs.DvsWeights(spec, wts, dev)
    frames = synth.dvs_frames(cfg_id, B, spec, stream=rank)
    x_dev = torch.from_numpy(frames).to(dev)
    gathered = torch.empty((world * B,), dtype=torch.int32, device=dev) if world > 1 else None
    stream = torch.cuda.current_stream(dev)

    def step(x):
        _, pred, _ = dvs_stages(dvs, spec, w, x, B)
        if world > 1:
            dist.all_gather_into_tensor(gathered, pred)
        return pred

    for _ in range(a.warmup):
        step(x_dev)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local, enabled=(rank == 0 and not a.no_clocks))
    clocks.start()
    # frames larger than L2 evict the previous step by themselves; smaller
    # ones get the 256 MiB flush write between steps, outside the events
    big = frames.nbytes > L2_BYTES
    flush = None if big else torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    times = []
    for _ in range(a.steps):
        if flush is not None:
            flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        step(x_dev)
        e1.record(stream)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    clk = clocks.stop()
    tot_ms = float(np.sum(times))
    if world > 1:
        t = torch.tensor([tot_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        tot_ms = float(t.item())
    value = world * B * a.steps / (tot_ms / 1e3)

    # end to end: pinned host frames -> device, the network, outputs back,
    # every step.  Frames larger than L2 go through dvs.run_host_batches
    # (step i+1's frames cross while step i computes); smaller ones step by
    # step through the same call with one batch, the L2 flush between steps.
    h_in = torch.from_numpy(frames).pin_memory()
    h_outs = [torch.empty((B, spec.classes), dtype=torch.float32).pin_memory() for _ in range(max(a.steps, 2))]
    h_preds = [torch.empty((B,), dtype=torch.int32).pin_memory() for _ in range(max(a.steps, 2))]
    dvs.run_host_batches(spec, w, [h_in] * 2, h_outs[:2], h_preds[:2])   # warms the copies
    torch.cuda.synchronize()
    if big:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        dvs.run_host_batches(spec, w, [h_in] * a.steps, h_outs[:a.steps], h_preds[:a.steps])
        e1.record(stream)
        torch.cuda.synchronize()
        e_times = [e0.elapsed_time(e1)]
    else:
        e_times = []
        for i in range(a.steps):
            flush.fill_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            dvs.run_host_batches(spec, w, [h_in], h_outs[i:i + 1], h_preds[i:i + 1])
            e1.record(stream)
            torch.cuda.synchronize()
            e_times.append(e0.elapsed_time(e1))
    e_ms = float(np.sum(e_times))
    if world > 1:
        t = torch.tensor([e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
    e2e = world * B * a.steps / (e_ms / 1e3)

    # per-stage roofline pass
    marks = []
    _, _, ev = dvs_stages(dvs, spec, w, x_dev, B, marks=marks)
    torch.cuda.synchronize()
    stage_ms = {}
    for name, e0, e1 in marks:
        stage_ms[name] = stage_ms.get(name, 0.0) + e0.elapsed_time(e1)
    alg = dvs_bytes(spec, B, ev)
    kern_ms = float(sum(stage_ms.values()))
    peak, peak_kind = peaks()
    achieved = alg / (kern_ms / 1e3) / 1e9
    conv1_bytes = 4 * B * spec.in_c * spec.H * spec.W * spec.T + 4 * B * spec.convs[0] * spec.H * spec.W
    res = None
    if rank == 0:
        res = {
            "metric": "images_per_sec", "value": round(value, 1), "unit": "samples/s",
            "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": round(tot_ms / a.steps, 4), "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic (seeded Bernoulli(0.05) event frames, Kaiming weights, see vdttfs/synth.py)",
            "config": {"workload": f"{netname} C{cfg_id}",
                       "model": f"dvs-culif {spec.in_c}x{spec.H}x{spec.W}, {spec.classes} classes",
                       "global_batch": world * B, "batch_per_gpu": B, "T": spec.T, "delta": spec.delta,
                       "parallelism": f"dp{world}",
                       "l2": (f"inputs larger than L2 (frames {frames.nbytes / B / 1e6:.1f} MB per sample)" if big
                              else "flushed (256 MiB write) between steps")},
            "e2e": {"value": round(e2e, 1), "unit": "samples/s", "h2d_bytes_per_step": int(frames.nbytes),
                    "d2h_bytes_per_step": int(B * spec.classes * 4 + B * 4),
                    "api": "dvs.run_host_batches (pipelined, frames > L2)" if big
                    else "dvs.run_host_batches one batch per step, L2 flushed between steps"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": None,
                         "kernel": "all DVS stages of one step", "peak_source": f"{peak_kind} hbm_gbs",
                         "algorithmic_bytes_per_step": int(alg), "kernel_ms_per_step": round(kern_ms, 4),
                         "stage_ms": {k: round(v, 4) for k, v in stage_ms.items()},
                         "conv1_gbs": round(conv1_bytes / (stage_ms["conv1_raw"] / 1e3) / 1e9, 1)},
            "gpu_launches": 13 * a.steps,
            "clocks": clk,
        }
        if not a.no_cpu_baseline:
            res["cpu_baseline"] = dvs_cpu_baseline(spec, wts, frames, budget_s=20.0)
    if world > 1:
        dist.destroy_process_group()
    return res


def dvs_cpu_baseline(spec, wts, frames, budget_s=20.0):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    cores = os.cpu_count() or 1
    n, reps, t_tot = 1, 0, 0.0
    while t_tot < budget_s * 0.5 and reps < 8:
        t0 = time.perf_counter()
        O.run_dvs(spec, wts, frames[:n])
        t_tot += time.perf_counter() - t0
        reps += 1
    return {"value": round(n * reps / t_tot, 3), "unit": "samples/s", "cores": cores, "kind": "port",
            "sample": f"{reps} passes of {n} sample of the same workload (full DVS network), "
                      f"OpenMP over {cores} threads"}


def run_dvs_reference(a):
    from vdttfs import nets, synth
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    netname, cfg_id, _, _, scaling = CONFIGS[a.config]
    spec = nets.dvs() if netname == "dvs" else nets.dvs_ref()
    wts = synth.dvs_weights(spec, cfg_id)
    n = 1
    frames = synth.dvs_frames(cfg_id, n, spec, stream=0)
    for _ in range(a.warmup):
        O.run_dvs(spec, wts, frames)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        O.run_dvs(spec, wts, frames)
    dt = time.perf_counter() - t0
    cores = os.cpu_count() or 1
    v = round(n * a.steps / dt, 3)
    return {"impl": "reference", "metric": "images_per_sec", "value": v, "unit": "samples/s",
            "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(dt / a.steps * 1e3, 3),
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
            "config": {"workload": f"{netname} C{cfg_id}", "batch_per_step": n, "T": spec.T, "delta": spec.delta},
            "cpu_baseline": {"value": v, "unit": "samples/s", "cores": cores, "kind": "port",
                             "sample": f"{n} sample per step, the CPU port of the reference's task-3 "
                                       f"path (oracle/vdt_oracle.c), OpenMP {cores} threads"},
            "e2e": {"value": v, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ------------------------------------------------- config 5: the sweep --
def sweep_point(E, nets, synth, dev, delta, zf, T, B, steps, warmup, flush):
    import torch
    net = nets.vgg16(T=T, delta=delta)
    layers = synth.kaiming_layers(net, 3)
    img = synth.images(5, B, net.in_h, net.in_w, net.in_c, zf)
    model = E.Model(net, layers, device=dev.index)
    ctx = E.Context(model, B)
    ctx.set_sub_batches(2)      # as the main workload
    x = torch.from_numpy(img).to(dev)
    ctx.set_counting(True)
    ctx.infer(x, pixels=True)
    torch.cuda.synchronize()
    events, fetched = ctx.counters()
    ctx.set_counting(False)
    for _ in range(warmup):
        ctx.infer(x, pixels=True)
    torch.cuda.synchronize()
    times = []
    for _ in range(steps):
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        ctx.infer(x, pixels=True)
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    ctx.set_profiling(True)
    ctx.layer_times()
    for _ in range(3):
        flush.fill_(1)
        ctx.infer(x, pixels=True)
    bkt, integ, pool, nb = ctx.layer_times()
    ctx.set_profiling(False)
    alg = sum(layer_bytes(net, layer_events(E, net, layers, x, B, dev), B))
    kern_ms = (float(np.sum(bkt)) + float(np.sum(integ))) / nb
    ms = float(np.mean(times))
    ctx.close()
    model.close()
    return {"delta": delta, "zero_frac": zf, "T": T, "images_per_sec": round(B / (ms / 1e3), 1),
            "ms_per_step": round(ms, 4), "integrator_gbs": round(alg / (kern_ms / 1e3) / 1e9, 1),
            "events_per_image": round(events / B, 1),
            "fetched_synapse_fraction": round(fetched / B / VGG16_DENSE_MACS, 4)}


def run_sweep(a):
    """VGG-16, batch 256, delta in {4,8,16,32,64} x input
    zero fraction in {0.2,0.5,0.9} x window T' in {80,40,20}.  delta sets the
    reference's bucket width and with it the fetched-synapse accounting; the
    engine's integrators are delta-invariant (k_sorted buckets at its own
    width), so images/s depends on the input and T' only."""
    import torch
    from vdttfs import engine as E, nets, synth
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    B = a.batch or 256
    pts = []
    for T in (80, 40, 20):
        for zf in (0.2, 0.5, 0.9):
            for delta in (4, 8, 16, 32, 64):
                pts.append(sweep_point(E, nets, synth, dev, delta, zf, T, B, a.steps, a.warmup, flush))
    head = next(p for p in pts if p["delta"] == 8 and p["zero_frac"] == 0.2 and p["T"] == 80)
    peak, peak_kind = peaks()
    return {"metric": "images_per_sec", "value": head["images_per_sec"], "unit": "images/s", "n_gpus": 1,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
            "config": {"workload": "vgg16 C5 sweep (value at delta 8, zero fraction 0.2, T 80)",
                       "batch_per_gpu": B, "l2": "flushed (256 MiB write) between steps"},
            "hbm_peak_gbs": peak, "peak_source": peak_kind, "sweep": pts}


def main():
    a = parse()
    if a.warmup < 3:
        a.warmup = 3
    if a.config == "vgg16_sweep":
        res = run_sweep(a)
    elif a.config in ("dvs", "dvs_ref"):
        res = run_dvs_reference(a) if a.impl == "reference" else run_dvs_engine(a)
    else:
        res = run_reference(a) if a.impl == "reference" else run_engine(a)
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
