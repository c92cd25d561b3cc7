"""Benchmark of the B200 VD-TTFS engine (one JSON line on rank 0).

Default workload: BASELINE config 3, the VGG-16 TTFS-SNN at batch 256 per GPU
(T=80, delta=8, TIME_FIRE_START=40), weak scaling over the GPUs of one box.
A step = one batch through the whole network (encode, 15 x {bucketize,
integrate}, 5 pools, membrane readout, argmax) + the NCCL all-gather of the
int32 predictions when N > 1.  The model uses the reference's host-libm LUTs
(built once at load), so its outputs are the reference's bit for bit.

  value   images/s over all ranks, input pixels already in HBM, device-timed
          with CUDA events per step (max over ranks); a 256 MiB L2-flush write
          runs between steps, outside the timed events.
  e2e     the same through the host entry points: pinned host pixels -> H2D
          -> the network -> D2H of the logits and predictions, every step
          (vdt_infer_host step by step with the L2 flush between steps; for a
          batch larger than L2, vdt_infer_host_batches, which overlaps step
          i+1's H2D copy with step i's compute).
  parity  the last timed step's outputs and predictions against the stored
          expected outputs of this batch (tests/golden/bench_parity.npz, from
          the oracle, which is pinned to the reference's kernels), and at one
          GPU against the reference's own kernels run on the same batch.
  roofline  the step's longest launch (its layer's integrator), timed live
          with CUDA events around each launch (eager profiling pass), against
          its implementation-independent algorithmic bytes (layer_bytes) and
          the measured HBM peak; beside it the same launch's FP32 FMA rate and
          weight-gather bandwidth against peaks measured on this GPU
          (vdt_measure_peaks), and the whole step's figures.
  ref_vdttfs_cuda  (one GPU) the reference's own vdttfs_cuda kernels and host
          helpers, compiled unmodified (oracle/_ref), on the same batch on the
          same GPU, timed the way its main times a batch.
  cpu_baseline  the CPU oracle port (OpenMP over all host cores) on a bounded
          sample of the same workload.

`--impl reference` times the reference algorithm's CPU implementation (the
oracle port; the reference ships no CPU implementation of this path) on the
same batch and prints its own line; under torchrun only rank 0 works.
`--baselines` runs, on one GPU, the reference's vdttfs_cuda batch for every
configuration it has and its step-by-step (time-driven) programs, and prints
one line with their throughputs (the reported baselines).
"""
import argparse
import gc
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
PARITY_FILE = os.path.join(ROOT, "tests", "golden", "bench_parity.npz")

CONFIGS = {
    # name: (net factory, config id, batch per GPU, zero fraction, scaling)
    "vgg16": ("vgg16", 3, 256, 0.0, "weak"),
    "lenet5": ("lenet5", 2, 65536, 0.8, "strong"),
    "lenet5_b1024": ("lenet5", 1, 1024, 0.8, "weak"),
    "dvs": ("dvs", 4, 64, 0.0, "weak"),     # task-3 CuLIF network, 2x128x128 event frames
    "dvs_ref": ("dvs_ref", 4, 64, 0.0, "weak"),   # the reference's own 2x32x32 DVS network
    "vgg16_sweep": ("vgg16", 5, 256, 0.2, "weak"),   # delta x zero fraction x T'
}
# reference task of each network (oracle/_ref/libref_t<task>.so)
REF_TASK = {"vgg16": 2, "lenet5": 1}

VGG16_DENSE_MACS = 313_725_952      # dense multiply-accumulates of one 3x32x32 VGG-16 image

# DRAM bytes (read + write) of one launch of the roofline's dominant kernel,
# from an ncu capture of that launch alone (dram__bytes_read.sum +
# dram__bytes_write.sum; command in the kernel's summary under profiles/),
# keyed by (workload, layer), with the commit of the build it measured.
DOMINANT_TRAFFIC = {
    ("vgg16", 1): (84_088_832 + 5_853_440, "k_dense conv1_2 at B=256 (its 2x2 pool fused in), kernels of build 70e92e0"),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="engine", choices=["engine", "reference"])
    ap.add_argument("--config", default="vgg16", choices=sorted(CONFIGS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ref-cuda", action="store_true", help="skip the reference vdttfs_cuda leg")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--baselines", action="store_true",
                    help="time the reference's vdttfs_cuda and step-by-step programs only")
    ap.add_argument("--batch", type=int, default=0,
                    help="override the config's batch (small cases for profiling; not a bench line)")
    ap.add_argument("--eager-once", action="store_true",
                    help="one eager batch (graphs off, one sub-batch, no counting) for a profiler; no bench line")
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
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
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


def probe_peaks(device):
    """FP32 FMA/s and L2 read bytes/s measured on this GPU now."""
    import ctypes as C
    from vdttfs._lib import check, lib
    f, l2 = C.c_double(), C.c_double()
    check(lib().vdt_measure_peaks(device, C.byref(f), C.byref(l2)), "vdt_measure_peaks")
    return f.value, l2.value


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
    """Kernel launches of one inference (graph path, one sub-batch): the
    pixel encoder unless the first layer runs k_dense (which encodes the
    pixels as it reads them); per layer its integrator, plus a bucketize pass unless the
    integrator reads the spike map itself (k_dense, k_thread, k_layer_vmem),
    plus a pool pass unless the pool runs fused into the integrator
    (k_thread, k_dense, k_sorted: everything but the generic chunk
    integrator); the readout unless the last layer is a membrane readout (it
    runs fused there).  Each sub-batch launches the same sequence.  The fused
    pools' pre-fill is a memset node, not a kernel."""
    from vdttfs.engine import KERNEL_CHUNK, KERNEL_DENSE, KERNEL_THREAD, KERNEL_VMEM
    n = 1 if pixels and kernels[0] != KERNEL_DENSE else 0
    for l, k in zip(net.layers, kernels):
        n += 1 if k in (KERNEL_DENSE, KERNEL_THREAD, KERNEL_VMEM) else 2
        n += 1 if l.pool_after and k == KERNEL_CHUNK else 0
    return n + (0 if kernels[-1] == KERNEL_VMEM else 1)


# ------------------------------------------------------------------ parity --
def stored_parity(config, out, pred, B):
    """The outputs / predictions of a step against the stored expected ones
    of this configuration's rank-0 batch: the configuration's own batch, or
    (strong scaling) rank 0's share of it, stored as "<config>@<B>"."""
    import hashlib
    try:
        g = np.load(PARITY_FILE)
    except Exception as e:
        return {"checked": False, "why": f"no stored outputs: {e}"}
    key = config if f"{config}_batch" in g.files and int(g[f"{config}_batch"]) == B else f"{config}@{B}"
    if f"{key}_batch" not in g.files:
        return {"checked": False, "why": f"no stored outputs for {config} at batch {B}"}
    out = np.ascontiguousarray(out, np.float32)
    digest_ok = hashlib.sha256(out.tobytes()).hexdigest() == str(g[f"{key}_out_sha256"])
    bad_pred = int(np.sum(np.asarray(pred, np.int32) != g[f"{key}_pred"].astype(np.int32)))
    return {"checked": True,
            "against": "expected outputs of this batch (oracle pinned to the reference's kernels), "
                       "tests/golden/bench_parity.npz",
            "out_sha256_equal": bool(digest_ok), "pred_differing": bad_pred, "images": B,
            "result": "bit-exact" if digest_ok and bad_pred == 0 else "MISMATCH"}


def live_parity(out, pred, r_out, r_pred):
    out = np.ascontiguousarray(out, np.float32).reshape(-1)
    r_out = np.ascontiguousarray(r_out, np.float32).reshape(-1)
    bad = int(np.sum(out.view(np.int32) != r_out.view(np.int32)))
    bad_pred = int(np.sum(np.asarray(pred).reshape(-1) != np.asarray(r_pred).reshape(-1)))
    return {"out_values_differing": bad, "pred_differing": bad_pred,
            "result": "bit-exact" if bad == 0 and bad_pred == 0 else "MISMATCH"}


# ------------------------------------------------------ reference on the GPU --
def ref_vdttfs_cuda(netname, cfg_id, net, layers, img, device, engine_out, engine_pred, reps=10,
                    clocks=True):
    """Reported baseline: the reference's own vdttfs_cuda batch (oracle/_ref,
    compiled unmodified from the reference sources) on this batch and GPU."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import refbind
    task = REF_TASK.get(netname)
    if task is None or not refbind.available(task):
        return {"unavailable": "no reference vdttfs_cuda program for this workload, or oracle/_ref not built"}
    import oracle as O
    spikes = O.encode_linear(img, net.T)
    ck = ClockSampler(device, enabled=clocks)
    ck.start()
    r = refbind.time_vdttfs_cuda(task, net, layers, spikes, reps=reps)
    clk = ck.stop()
    B = img.shape[0]
    return {"value": round(B / (r["ms_per_batch"] / 1e3), 1), "unit": "images/s", "batch": B, "reps": reps,
            "ms_per_batch": round(r["ms_per_batch"], 4),
            "timing": "CUDA events around reps batches, each: H2D of the spike times, every layer through the "
                      "reference's host helpers (update_LUTs with blocking copies, a device sync after every "
                      "launch), D2H of the outputs, host readout",
            "program": f"oracle/_ref/libref_t{task}.so (the reference's vdttfs_cuda program, unmodified)",
            "parity_vs_engine": live_parity(engine_out, engine_pred, r["out"], r["pred"]),
            "clocks": clk}


def ref_dvs_cuda(spec, wts, frames, device, engine_out, engine_pred, reps=10, clocks=True):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import refbind
    if spec.H != 32 or spec.W != 32 or not refbind.available(3):
        return {"unavailable": "the reference's task-3 kernels are hard-coded to 2x32x32 input "
                               "(the dvs_ref workload), or oracle/_ref not built"}
    ck = ClockSampler(device, enabled=clocks)
    ck.start()
    r = refbind.time_dvs_ref(spec, wts, frames, reps=reps)
    clk = ck.stop()
    B = frames.shape[0]
    return {"value": round(B / (r["ms_per_batch"] / 1e3), 1), "unit": "samples/s", "batch": B, "reps": reps,
            "ms_per_batch": round(r["ms_per_batch"], 4),
            "timing": "CUDA events around reps batches of the reference's seven stages and four "
                      "bucketizations on device-resident frames, output copied back",
            "program": "oracle/_ref/libref_t3.so (the reference's task-3 kernels, unmodified)",
            "parity_vs_engine": live_parity(engine_out, engine_pred, r["out"], r["pred"]),
            "clocks": clk}


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
    model = E.Model(net, layers, device=local, lut_source=E.LUT_HOST_LIBM)
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

    # ---- counters (per-layer events / fetched synapses) on one untimed batch
    ctx.set_counting(True)
    with torch.cuda.stream(stream):
        ctx.infer(x_dev, pixels=True, out=out, pred=pred)
    stream.synchronize()
    ev_layer, fe_layer = ctx.layer_counters()
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
    evs = timing_events(torch, a.steps)
    gc.disable()                      # no collector pauses of this harness inside the timed steps
    for e0, e1 in evs:
        with torch.cuda.stream(stream):
            flush.fill_(1)
            e0.record(stream)
            step()
            e1.record(stream)
        stream.synchronize()
        times.append(e0.elapsed_time(e1))
    gc.enable()
    clk = clocks.stop()
    tot_ms = float(np.sum(times))
    if world > 1:
        t = torch.tensor([tot_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        tot_ms = float(t.item())
    value = world * B * a.steps / (tot_ms / 1e3)
    step_out, step_pred = out.cpu().numpy(), pred.cpu().numpy()      # the last timed step's results

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
        e2e_out, e2e_pred = h_outs[a.steps - 1].numpy(), h_preds[a.steps - 1].numpy()
    else:
        h_out = torch.empty((B, net.n_classes), dtype=torch.float32).pin_memory()
        h_pred = torch.empty((B,), dtype=torch.int32).pin_memory()
        for _ in range(max(1, a.warmup)):
            ctx.infer_host(h_in, pixels=True, out=h_out, pred=h_pred)
        if world > 1:
            dist.barrier()
        e_times = []
        evs = timing_events(torch, a.steps)
        gc.disable()
        for e0, e1 in evs:
            with torch.cuda.stream(stream):
                flush.fill_(1)
                e0.record(stream)
            ctx.infer_host(h_in, pixels=True, out=h_out, pred=h_pred)
            with torch.cuda.stream(stream):
                e1.record(stream)
            stream.synchronize()
            e_times.append(e0.elapsed_time(e1))
        gc.enable()
        e2e_out, e2e_pred = h_out.numpy(), h_pred.numpy()
    e_ms = float(np.sum(e_times))
    if world > 1:
        t = torch.tensor([e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
    e2e = world * B * a.steps / (e_ms / 1e3)

    # ---- roofline: per-launch CUDA events (eager profiling pass, after one
    # untimed eager batch: the first eager launches carry one-off costs)
    ctx.set_profiling(True)
    with torch.cuda.stream(stream):
        ctx.infer(x_dev, pixels=True, out=out, pred=pred)
    stream.synchronize()
    ctx.layer_times()
    prof_steps = max(3, min(a.steps, 10))
    for _ in range(prof_steps):
        with torch.cuda.stream(stream):
            flush.fill_(1)
            ctx.infer(x_dev, pixels=True, out=out, pred=pred)
    bkt_ms, int_ms, pool_ms, nb = ctx.layer_times()
    ctx.set_profiling(False)
    kernels = ctx.layer_kernels()
    lbytes = layer_bytes(net, ev_layer, B)
    bkt_l, int_l = np.asarray(bkt_ms) / nb, np.asarray(int_ms) / nb
    dom = int(np.argmax(int_l))                                       # the step's longest launch
    dom_ms = float(int_l[dom])
    hbm_peak, peak_kind = peaks()
    dom_gbs = lbytes[dom] / (dom_ms / 1e3) / 1e9
    work_ms = float(bkt_l.sum() + int_l.sum())
    fma_peak, l2_peak = probe_peaks(local)
    dom_fma = fe_layer[dom] / (dom_ms / 1e3)
    step_fma = sum(fe_layer) / (work_ms / 1e3)
    traffic = DOMINANT_TRAFFIC.get((netname, dom)) if B == 256 else None

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
                       "sub_batches": 2, "luts": "host libm (the reference's tables)"},
            "e2e": {"value": round(e2e, 1), "unit": "images/s",
                    "h2d_bytes_per_step": int(img.nbytes),
                    "d2h_bytes_per_step": int(B * net.n_classes * 4 + B * 4),
                    "api": "vdt_infer_host_batches (pipelined, batch > L2)" if pipelined
                    else "vdt_infer_host per step, L2 flushed between steps",
                    "step_ms": step_spread(e_times, a.steps)},
            "parity": stored_parity(a.config, step_out, step_pred, B) if not a.batch else {"checked": False},
            "roofline": {
                "bound": "hbm", "achieved": round(dom_gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                "frac": round(dom_gbs / hbm_peak, 4),
                "traffic": None if traffic is None else int(traffic[0]),
                "traffic_source": None if traffic is None else
                "ncu dram__bytes_read.sum + dram__bytes_write.sum of this launch alone, " + traffic[1],
                "kernel": f"{E.KERNEL_NAMES[kernels[dom]]}, layer {dom} (the step's longest launch)",
                "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)",
                "algorithmic_bytes_per_launch": int(lbytes[dom]), "launch_ms": round(dom_ms, 4),
                "limiter": "not HBM: every fetched synapse is one 4-byte weight read from L1/L2 and one FP32 "
                           "FMA in a per-neuron chain of fixed order; the weights and bucket lists stay in L2",
                "fp32_fma": {"achieved_per_s": round(dom_fma / 1e12, 3), "peak_per_s": round(fma_peak / 1e12, 3),
                             "unit": "TFMA/s", "frac": round(dom_fma / fma_peak, 4),
                             "fetched_synapses": int(fe_layer[dom]),
                             "peak_source": "measured now on this GPU (vdt_measure_peaks: packed fma.rn.f32x2 "
                                            "chains on every SM)"},
                "weight_gather": {"achieved_gbs": round(4 * fe_layer[dom] / (dom_ms / 1e3) / 1e9, 1),
                                  "l2_read_peak_gbs": round(l2_peak / 1e9, 1),
                                  "frac": round(4 * fe_layer[dom] / (dom_ms / 1e3) / l2_peak, 4),
                                  "bytes": int(4 * fe_layer[dom]),
                                  "peak_source": "measured now on this GPU (vdt_measure_peaks: 16-byte L2-only "
                                                 "loads of a 32 MiB resident buffer); hits in L1 are counted too"},
                "step": {"algorithmic_bytes": int(sum(lbytes)), "kernel_ms": round(work_ms, 4),
                         "hbm_gbs": round(sum(lbytes) / (work_ms / 1e3) / 1e9, 1),
                         "hbm_frac": round(sum(lbytes) / (work_ms / 1e3) / 1e9 / hbm_peak, 4),
                         "fp32_fma_frac": round(step_fma / fma_peak, 4),
                         "integrate_ms_per_layer": [round(float(v), 4) for v in int_l],
                         "bucketize_ms": round(float(bkt_l.sum()), 4),
                         "pool_ms": round(float(np.sum(pool_ms)) / nb, 4),
                         "algorithmic_bytes_per_layer": [int(v) for v in lbytes],
                         "fetched_synapses_per_layer": [int(v) for v in fe_layer],
                         "kernels": [f"L{i}:{E.KERNEL_NAMES[k]}" for i, k in enumerate(kernels)]}},
            "gpu_launches": launches_per_step(net, kernels) * 2 * a.steps,     # two sub-batches per step
            "events_per_image": round(sum(ev_layer) / B, 1),
            "fetched_synapses_per_image": round(sum(fe_layer) / B, 1),
            "clocks": clk,
        }
        res["e2e"]["parity_vs_device_step"] = live_parity(e2e_out, e2e_pred, step_out, step_pred)["result"]
        if world == 1 and not a.no_ref_cuda and not a.batch:
            r = ref_vdttfs_cuda(netname, cfg_id, net, layers, img, local, step_out, step_pred,
                                clocks=not a.no_clocks)
            if "value" in r:
                r["engine_e2e_over_ref"] = round(e2e / r["value"], 3)
                r["engine_value_over_ref"] = round(value / r["value"], 3)
            res["ref_vdttfs_cuda"] = r
        if not a.no_cpu_baseline:
            res["cpu_baseline"] = cpu_baseline(net, layers, img, cfg_id, budget_s=20.0)
    if world > 1:
        del ctx
        dist.destroy_process_group()
    return res


# --------------------------------------------------------------- CPU legs --
def timing_events(torch, n):
    """n (start, stop) CUDA timing event pairs, made before a timed loop."""
    return [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]


def step_spread(times_ms, steps):
    """min / median / max of the per-step times (one pipelined call over all
    steps gives only its mean)."""
    t = np.asarray(times_ms, np.float64)
    if t.size == 1 and steps > 1:
        return {"mean": round(float(t[0]) / steps, 4)}
    return {"min": round(float(t.min()), 4), "median": round(float(np.median(t)), 4),
            "max": round(float(t.max()), 4)}


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


# images per step of the reference arm: the whole batch where the CPU port
# gets through the run in a few minutes, else a bounded sample of it
REF_ARM_IMAGES = {"vgg16": 256, "lenet5_b1024": 1024, "lenet5": 8192}


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
    n = min(REF_ARM_IMAGES.get(a.config, Bcfg), a.batch or Bcfg)
    img = synth.images(cfg_id, n, net.in_h, net.in_w, net.in_c, zf, stream=0)
    for _ in range(a.warmup):
        O.run_net(net, layers, O.encode_linear(img, net.T))
    t0 = time.perf_counter()
    for _ in range(a.steps):
        O.run_net(net, layers, O.encode_linear(img, net.T))
    dt = time.perf_counter() - t0
    v = round(n * a.steps / dt, 2)
    same = n == Bcfg
    return {"impl": "reference", "metric": "images_per_sec", "value": v, "unit": "images/s",
            "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": round(dt / a.steps * 1e3, 3), "higher_is_better": True, "scaling": scaling,
            "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
            "config": {"workload": f"{netname} C{cfg_id}", "model": netname, "batch_per_gpu": n,
                       "T": net.T, "delta": net.delta, "same_batch_as_engine": same},
            "cpu_baseline": {"value": v, "unit": "images/s", "cores": cores, "kind": "port",
                             "sample": (f"the engine's whole batch ({n} images, rank 0's) per step" if same else
                                        f"{n} of the batch's {Bcfg} images per step") +
                                       ", the CPU port of the reference's vdttfs algorithm (oracle/vdt_oracle.c), "
                                       f"OpenMP {cores} threads"},
            "e2e": {"value": v, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ------------------------------------------------------------ DVS (task 3) --
def dvs_bytes(spec, N, ev_rows):
    """Algorithmic bytes of one DVS batch: every stage's input map read and
    output map written once (conv1: the dense frames), the bucketed stages'
    lists written and read back (8 B per kept event, 4 B per chunk offset;
    none for a conv that reads its input map itself), the weights once.
    ev_rows: kept events of the FC1 and FC2 inputs."""
    s = spec.stage_shapes()
    c1n, c2n, c3n = spec.convs
    HW, HW2, HW4 = spec.H * spec.W, spec.H * spec.W // 4, spec.H * spec.W // 16
    OS = spec.n_chunks + 1
    k2 = spec.k * spec.k
    lists = lambda E, cols: 2 * (8 * E + 4 * cols * OS)
    b = 4 * N * spec.in_c * HW * spec.T + 4 * N * c1n * HW + 4 * c1n * spec.in_c * k2          # conv1
    b += 4 * N * c1n * HW + 4 * N * c2n * HW + 4 * c2n * c1n * k2                               # conv2 (fused)
    b += 4 * N * c2n * HW + 4 * N * c2n * HW2                                                    # pool1
    b += 4 * N * c2n * HW2 + 4 * N * c3n * HW2 + 4 * c3n * c2n * k2                              # conv3 (fused)
    b += 4 * N * c3n * HW2 + 4 * N * c3n * HW4                                                   # pool2
    b += 4 * N * s["fc1_in"] + 4 * N * spec.hidden + lists(ev_rows[0], N) + 4 * s["fc1_in"] * spec.hidden \
        + 4 * spec.hidden * spec.hidden                                                         # fc1
    b += 4 * N * spec.hidden + 4 * N * spec.classes + lists(ev_rows[1], N) + 4 * spec.hidden * spec.classes
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
    net = dvs.DvsNet(spec, wts, device=local)                 # the flat blob through vdt_model_load_dvs_flat
    stream = torch.cuda.Stream(device=dev)
    ctx = net.context(B, stream=stream.cuda_stream)
    frames = synth.dvs_frames(cfg_id, B, spec, stream=rank)
    x_dev = torch.from_numpy(frames).to(dev)
    out = torch.empty((B, spec.classes), dtype=torch.float32, device=dev)
    pred = torch.empty((B,), dtype=torch.int32, device=dev)
    gathered = torch.empty((world * B,), dtype=torch.int32, device=dev) if world > 1 else None

    def step():
        ctx.infer(x_dev, out=out, pred=pred)
        if world > 1:
            with torch.cuda.stream(stream):
                dist.all_gather_into_tensor(gathered, pred)

    for _ in range(a.warmup):
        with torch.cuda.stream(stream):
            step()
    stream.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local, enabled=(rank == 0 and not a.no_clocks))
    clocks.start()
    # frames larger than L2 evict the previous step by themselves; smaller
    # ones get the 256 MiB flush write between steps, outside the events
    big = frames.nbytes > L2_BYTES
    flush = None if big else torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    times = []
    evs = timing_events(torch, a.steps)
    gc.disable()
    for e0, e1 in evs:
        with torch.cuda.stream(stream):
            if flush is not None:
                flush.fill_(1)
            e0.record(stream)
            step()
            e1.record(stream)
        stream.synchronize()
        times.append(e0.elapsed_time(e1))
    gc.enable()
    clk = clocks.stop()
    tot_ms = float(np.sum(times))
    if world > 1:
        t = torch.tensor([tot_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        tot_ms = float(t.item())
    value = world * B * a.steps / (tot_ms / 1e3)
    step_out, step_pred = out.cpu().numpy(), pred.cpu().numpy()

    # end to end: pinned host frames -> device, the network, outputs back,
    # every step, through the C runtime's host calls.  Frames larger than L2
    # go through vdt_infer_host_batches (step i+1's frames cross while step i
    # computes); smaller ones through vdt_infer_host, the L2 flush between steps.
    h_in = torch.from_numpy(frames).pin_memory()
    h_outs = [torch.empty((B, spec.classes), dtype=torch.float32).pin_memory() for _ in range(max(a.steps, 2))]
    h_preds = [torch.empty((B,), dtype=torch.int32).pin_memory() for _ in range(max(a.steps, 2))]
    ctx.infer_host_batches([h_in] * 2, outs=h_outs[:2], preds=h_preds[:2])   # both slots' graphs
    if world > 1:
        dist.barrier()
    if big:
        with torch.cuda.stream(stream):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        ctx.infer_host_batches([h_in] * a.steps, outs=h_outs[:a.steps], preds=h_preds[:a.steps])
        with torch.cuda.stream(stream):
            e1.record(stream)
        stream.synchronize()
        e_times = [e0.elapsed_time(e1)]
    else:
        e_times = []
        evs = timing_events(torch, a.steps)
        gc.disable()
        for i, (e0, e1) in enumerate(evs):
            with torch.cuda.stream(stream):
                flush.fill_(1)
                e0.record(stream)
            ctx.infer_host(h_in, out=h_outs[i], pred=h_preds[i])
            with torch.cuda.stream(stream):
                e1.record(stream)
            stream.synchronize()
            e_times.append(e0.elapsed_time(e1))
        gc.enable()
    e_ms = float(np.sum(e_times))
    if world > 1:
        t = torch.tensor([e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
    e2e = world * B * a.steps / (e_ms / 1e3)
    e2e_out, e2e_pred = h_outs[a.steps - 1].numpy(), h_preds[a.steps - 1].numpy()

    # per-stage roofline pass (profiling: CUDA events around every stage),
    # after one untimed eager batch
    ctx.set_profiling(True)
    with torch.cuda.stream(stream):
        ctx.infer(x_dev, out=out, pred=pred)
    stream.synchronize()
    ctx.layer_times()
    prof_steps = 3
    for _ in range(prof_steps):
        with torch.cuda.stream(stream):
            if flush is not None:
                flush.fill_(1)
            ctx.infer(x_dev, out=out, pred=pred)
    bkt, comp, nb = ctx.layer_times()
    ctx.set_profiling(False)
    stage_ms = {n: round(float(b + c) / nb, 4) for n, b, c in zip(dvs.DvsNet.STAGES, bkt, comp)}
    ev_rows = dvs_row_events(dvs, spec, ctx, x_dev)
    alg = dvs_bytes(spec, B, ev_rows)
    kern_ms = float(sum(stage_ms.values()))
    peak, peak_kind = peaks()
    conv1_bytes = 4 * B * spec.in_c * spec.H * spec.W * spec.T + 4 * B * spec.convs[0] * spec.H * spec.W
    conv1_gbs = conv1_bytes / (stage_ms["conv1"] / 1e3) / 1e9
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
                    "api": "vdt_infer_host_batches (pipelined, frames > L2)" if big
                    else "vdt_infer_host per step, L2 flushed between steps",
                    "step_ms": step_spread(e_times, a.steps),
                    "parity_vs_device_step": live_parity(e2e_out, e2e_pred, step_out, step_pred)["result"]},
            "parity": stored_parity(a.config, step_out, step_pred, B) if not a.batch else {"checked": False},
            "roofline": {"bound": "hbm", "achieved": round(conv1_gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(conv1_gbs / peak, 4), "traffic": None,
                         "kernel": "k_culif_conv1 (the step's longest stage: dense frame read)",
                         "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)",
                         "algorithmic_bytes_per_launch": int(conv1_bytes), "launch_ms": stage_ms["conv1"],
                         "step": {"algorithmic_bytes": int(alg), "kernel_ms": round(kern_ms, 4),
                                  "hbm_gbs": round(alg / (kern_ms / 1e3) / 1e9, 1),
                                  "hbm_frac": round(alg / (kern_ms / 1e3) / 1e9 / peak, 4),
                                  "stage_ms": stage_ms}},
            "gpu_launches": 11 * a.steps,      # conv1, conv2, pool1, conv3, pool2, 3 for FC1, 2 for FC2, readout
            "clocks": clk,
        }
        if world == 1 and not a.no_ref_cuda and not a.batch:
            r = ref_dvs_cuda(spec, wts, frames, local, step_out, step_pred, clocks=not a.no_clocks)
            if "value" in r:
                r["engine_e2e_over_ref"] = round(e2e / r["value"], 3)
                r["engine_value_over_ref"] = round(value / r["value"], 3)
            res["ref_vdttfs_cuda"] = r
        if not a.no_cpu_baseline:
            res["cpu_baseline"] = dvs_cpu_baseline(spec, wts, frames, budget_s=20.0)
    ctx.close()
    net.close()
    if world > 1:
        dist.destroy_process_group()
    return res


def dvs_row_events(dvs, spec, ctx, x_dev):
    """Kept events of the FC1 and FC2 inputs (the bucketed stages), from the
    engine's own bucketing of the traced pool2 and fc1 maps."""
    maps, _, _ = ctx.trace(x_dev)
    N = x_dev.shape[0]
    s = dvs.internal_spec(spec)
    e = []
    for m, F in ((maps[4], spec.stage_shapes()["fc1_in"]), (maps[5], spec.hidden)):
        off, _, _ = dvs.bucketize_rows(m, N, F, s)
        e.append(int(off[:, -1].sum().item()))
    return e


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
    netname, cfg_id, Bcfg, _, scaling = CONFIGS[a.config]
    spec = nets.dvs() if netname == "dvs" else nets.dvs_ref()
    wts = synth.dvs_weights(spec, cfg_id)
    n = 1 if netname == "dvs" else Bcfg           # a 2x128x128 sample takes the port about a second
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
            "config": {"workload": f"{netname} C{cfg_id}", "batch_per_gpu": n, "T": spec.T, "delta": spec.delta,
                       "same_batch_as_engine": n == Bcfg},
            "cpu_baseline": {"value": v, "unit": "samples/s", "cores": cores, "kind": "port",
                             "sample": f"{n} sample(s) per step, the CPU port of the reference's task-3 "
                                       f"path (oracle/vdt_oracle.c), OpenMP {cores} threads"},
            "e2e": {"value": v, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ------------------------------------------------- config 5: the sweep --
def sweep_point(E, nets, synth, dev, delta, zf, T, B, steps, warmup, flush):
    import torch
    net = nets.vgg16(T=T, delta=delta)
    layers = synth.kaiming_layers(net, 3)
    img = synth.images(5, B, net.in_h, net.in_w, net.in_c, zf)
    model = E.Model(net, layers, device=dev.index, lut_source=E.LUT_HOST_LIBM)
    ctx = E.Context(model, B)
    ctx.set_sub_batches(2)      # as the main workload
    x = torch.from_numpy(img).to(dev)
    ctx.set_counting(True)
    ctx.infer(x, pixels=True)
    torch.cuda.synchronize()
    ev_layer, fe_layer = ctx.layer_counters()
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
    alg = sum(layer_bytes(net, ev_layer, B))
    kern_ms = (float(np.sum(bkt)) + float(np.sum(integ))) / nb
    ms = float(np.mean(times))
    ctx.close()
    model.close()
    return {"delta": delta, "zero_frac": zf, "T": T, "images_per_sec": round(B / (ms / 1e3), 1),
            "ms_per_step": round(ms, 4), "integrator_gbs": round(alg / (kern_ms / 1e3) / 1e9, 1),
            "events_per_image": round(sum(ev_layer) / B, 1),
            "fetched_synapse_fraction": round(sum(fe_layer) / B / VGG16_DENSE_MACS, 4)}


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


# ------------------------------------------------ the reported baselines --
def run_baselines(a):
    """The reference's own GPU programs on one GPU (rank 0): its vdttfs_cuda
    batch on every bench workload it has a program for, then its
    step-by-step (time-driven) programs, each on seeded synthetic inputs."""
    import torch
    from vdttfs import nets, synth
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    import refbind
    torch.cuda.set_device(0)
    res = {"impl": "reference GPU programs (reported baselines)", "vdttfs_cuda": {}, "stepbystep_cuda": {}}
    for config in ("vgg16", "lenet5_b1024", "lenet5"):
        netname, cfg_id, B, zf, _ = CONFIGS[config]
        net = nets.NETS[netname]()
        layers = synth.kaiming_layers(net, cfg_id)
        img = synth.images(cfg_id, B, net.in_h, net.in_w, net.in_c, zf, stream=0)
        ck = ClockSampler(0, enabled=not a.no_clocks)
        ck.start()
        r = refbind.time_vdttfs_cuda(REF_TASK[netname], net, layers, O.encode_linear(img, net.T))
        clk = ck.stop()
        res["vdttfs_cuda"][config] = {"images_per_sec": round(B / (r["ms_per_batch"] / 1e3), 1), "batch": B,
                                      "ms_per_batch": round(r["ms_per_batch"], 4),
                                      "parity": stored_parity(config, r["out"], r["pred"], B), "clocks": clk}
    spec = nets.dvs_ref()
    frames = synth.dvs_frames(4, 64, spec, stream=0)
    r = refbind.time_dvs_ref(spec, synth.dvs_weights(spec, 4), frames)
    res["vdttfs_cuda"]["dvs_ref"] = {"samples_per_sec": round(64 / (r["ms_per_batch"] / 1e3), 1), "batch": 64,
                                     "ms_per_batch": round(r["ms_per_batch"], 4),
                                     "parity": stored_parity("dvs_ref", r["out"], r["pred"], 64)}
    for prog in ("vgg16", "vgg16_lut", "lenet_ref"):
        ck = ClockSampler(0, enabled=not a.no_clocks)
        ck.start()
        r = refbind.run_stepbystep(prog)
        r["clocks"] = ck.stop()
        res["stepbystep_cuda"][prog] = r
    return res


def run_eager_once(a):
    """One batch of the configuration through the engine without graphs or
    sub-batches, each layer's launches in layer order: the program a
    profiler captures single launches of (ncu -k / -s / -c)."""
    import torch
    from vdttfs import engine as E, nets, synth
    netname, cfg_id, Bcfg, zf, _ = CONFIGS[a.config]
    net = nets.NETS[netname]()
    B = a.batch or Bcfg
    m = E.Model(net, synth.kaiming_layers(net, cfg_id), lut_source=E.LUT_HOST_LIBM)
    ctx = E.Context(m, B, graphs=False)
    x = torch.from_numpy(synth.images(cfg_id, B, net.in_h, net.in_w, net.in_c, zf, stream=0)).cuda()
    out, pred = ctx.infer(x, pixels=True)
    torch.cuda.synchronize()
    print("eager batch", a.config, B, ctx.layer_kernels(), flush=True)
    return None


def main():
    a = parse()
    if a.warmup < 3:
        a.warmup = 3
    if a.eager_once:
        res = run_eager_once(a)
    elif a.baselines:
        res = run_baselines(a)
    elif a.config == "vgg16_sweep":
        res = run_sweep(a)
    elif a.config in ("dvs", "dvs_ref"):
        res = run_dvs_reference(a) if a.impl == "reference" else run_dvs_engine(a)
    else:
        res = run_reference(a) if a.impl == "reference" else run_engine(a)
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
