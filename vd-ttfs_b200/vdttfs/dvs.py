"""Task 3 (DVS gesture) on the engine: the reference's CuLIF stages
(task3_dvsgesture/vdttfs_cuda/snn_inference_timesorted.cu, "t3") as device
calls through the C ABI, and the per-batch pipeline of its main.

  conv1_raw        conv1_raw_early        t3:30-65
  bucketize        k_bucketize_conv/fc    t3:70-106   (VDT_TB_TRUNC)
  conv_bucketed    conv_bucketed_early    t3:109-143
  pool             pool_chunk_early       t3:146-168
  fc1_recurrent    fc1_bucketed_recurrent t3:171-200
  fc2              fc2_bucketed_early     t3:203-225
  readout          argmin, lowest index   t3:295-296

Maps are NCHW fp32 spike times as in the reference.  Weights arrive in the
reference's layouts (OIHW convs, [out, in] FC, [hidden, hidden] recurrent)
and are permuted once on the device (DvsWeights).
"""
from __future__ import annotations

import ctypes as C
import dataclasses
import weakref

import numpy as np

from . import nets
from ._lib import DvsDesc, TimeCfg, check, lib
from .engine import LAYOUT_NCHW, LAYOUT_NHWC, TB_TRUNC, Context, _ptr, _stream, bucketize, readout


def _cfg(spec: nets.DvsSpec) -> TimeCfg:
    return TimeCfg(spec.T, spec.delta, 0.0, 1.0, 9999.0, nets.LUT_BY_TB, spec.T, 0)


class DvsWeights:
    """Device copies of a DVS network's weights in the kernels' layouts."""

    def __init__(self, spec: nets.DvsSpec, wts: dict, device="cuda"):
        import torch
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(device)
        self.spec = spec
        self.conv1 = t(wts["conv1"])                           # OIHW, read as is
        self.conv2 = oihw_to_hwio(t(wts["conv2"]))
        self.conv3 = oihw_to_hwio(t(wts["conv3"]))
        self.fc1_t = t(np.asarray(wts["fc1"]).T)                # [F_in, hidden]
        self.rec_t = t(np.asarray(wts["fc1_rec"]).T)            # [hidden, hidden], [j][i]
        self.fc2_t = t(np.asarray(wts["fc2"]).T)                # [hidden, classes]


def dvs_desc(spec: nets.DvsSpec) -> DvsDesc:
    """The C ABI's vdt_dvs_desc of a network spec."""
    c1, c2, c3 = spec.convs
    return DvsDesc(spec.in_c, spec.H, spec.W, spec.T, spec.delta, c1, c2, c3, spec.k, spec.hidden,
                   spec.classes, spec.decay_conv, spec.th_conv, spec.decay_fc, spec.th_fc)


class DvsNet:
    """The whole task-3 network as one engine model: the reference's flat
    weight blob (t3:237-241; `weights` is the blob's bytes or the dict of
    synth.dvs_weights / assets.load_dvs_flat) loaded by
    vdt_model_load_dvs_flat, run per batch by the C++ runtime (one captured
    CUDA graph per batch size, workspace owned by the context)."""

    STAGES = ("conv1", "conv2", "pool1", "conv3", "pool2", "fc1", "fc2")

    def __init__(self, spec: nets.DvsSpec, weights, device: int = 0):
        from .assets import write_dvs_flat
        self.spec = spec
        blob = bytes(weights) if isinstance(weights, (bytes, bytearray, memoryview)) else write_dvs_flat(weights, spec)
        self._desc = dvs_desc(spec)
        h = C.c_void_p()
        check(lib().vdt_model_load_dvs_flat(blob, len(blob), C.byref(self._desc), device, C.byref(h)),
              "vdt_model_load_dvs_flat")
        self.h = h
        self.device = device
        self.n_classes = spec.classes
        self._contexts = weakref.WeakSet()

    def context(self, max_batch: int, stream=None, graphs: bool = True) -> "DvsContext":
        return DvsContext(self, max_batch, stream=stream, graphs=graphs)

    def stage_shapes(self, N: int):
        s = self.spec
        c1, c2, c3 = s.convs
        return [(N, c1, s.H, s.W), (N, c2, s.H, s.W), (N, c2, s.H // 2, s.W // 2), (N, c3, s.H // 2, s.W // 2),
                (N, c3, s.H // 4, s.W // 4), (N, s.hidden), (N, s.classes)]

    def close(self):
        if self.h:
            for c in list(self._contexts):
                c.close()
            lib().vdt_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DvsContext(Context):
    """Per-stream workspace of a DvsNet.  infer / infer_host /
    infer_host_batches take frames [N, C, H, W, T] (time innermost) and return
    FC2's first-spike times [N, classes] and the argmin readout."""

    def layer_times(self):
        """Per stage (DvsNet.STAGES) the bucketize and compute milliseconds
        accumulated since the last call, and the number of batches."""
        n = len(DvsNet.STAGES)
        a, b, c = (np.zeros(n, np.float32) for _ in range(3))
        nb = C.c_int()
        check(lib().vdt_ctx_layer_times(self.h, n, a.ctypes.data, b.ctypes.data, c.ctypes.data,
                                        C.byref(nb)), "vdt_ctx_layer_times")
        return a, b, nb.value

    def layer_kernels(self):
        """Raises VdtError (VDT_ERR_UNSUPPORTED): the stages' kernels are fixed."""
        k = np.zeros(len(DvsNet.STAGES), np.int32)
        check(lib().vdt_ctx_layer_kernels(self.h, len(k), k.ctypes.data), "vdt_ctx_layer_kernels")
        return [int(v) for v in k]

    def trace(self, frames):
        """The whole network, returning every stage's output map."""
        import torch
        N = frames.shape[0]
        maps = [torch.empty(s, dtype=torch.float32, device=frames.device) for s in self.model.stage_shapes(N)]
        arr = (C.c_void_p * len(maps))(*[_ptr(m) for m in maps])
        out = torch.empty((N, self.model.n_classes), dtype=torch.float32, device=frames.device)
        pred = torch.empty((N,), dtype=torch.int32, device=frames.device)
        check(lib().vdt_infer_trace(self.h, _ptr(frames), 0, N, arr, _ptr(out), _ptr(pred)), "vdt_infer_trace")
        return maps, out, pred


def oihw_to_hwio(w, stream=None):
    import torch
    O, I, K, _ = w.shape
    out = torch.empty((K, K, I, O), dtype=torch.float32, device=w.device)
    check(lib().vdt_oihw_to_hwio(_ptr(w), _ptr(out), O, I, K, C.c_void_p(_stream(stream))), "vdt_oihw_to_hwio")
    return out


def conv1_raw(frames, w_oihw, spec: nets.DvsSpec, stream=None):
    import torch
    N = frames.shape[0]
    c1 = spec.convs[0]
    out = torch.empty((N, c1, spec.H, spec.W), dtype=torch.float32, device=frames.device)
    check(lib().vdt_dvs_conv1_raw(_ptr(frames), _ptr(w_oihw), N, spec.in_c, c1, spec.H, spec.W, spec.k,
                                  spec.T, spec.delta, spec.decay_conv, spec.th_conv, _ptr(out),
                                  C.c_void_p(_stream(stream))), "vdt_dvs_conv1_raw")
    return out


def bucketize_sites(x, N, C_in, H, W, spec, stream=None):
    """Buckets of an NCHW map, one column per site (k_bucketize_conv)."""
    return bucketize(x.reshape(-1), N * H * W, C_in, _cfg(spec), layout=LAYOUT_NCHW, hw=H * W,
                     tb_mode=TB_TRUNC, stream=stream)


def bucketize_rows(x, N, F, spec, stream=None):
    """Buckets of [N, F] feature rows (k_bucketize_fc)."""
    return bucketize(x.reshape(-1), N, F, _cfg(spec), layout=LAYOUT_NHWC, hw=1, tb_mode=TB_TRUNC,
                     stream=stream)


def conv_bucketed(buckets, w_hwio, N, C_in, C_out, H, W, spec, out_layout=LAYOUT_NCHW, stream=None):
    import torch
    off, cin, tin = buckets
    out = torch.empty((N * C_out * H * W,), dtype=torch.float32, device=off.device)
    check(lib().vdt_dvs_conv_bucketed(_ptr(off), _ptr(cin), _ptr(tin), _ptr(w_hwio), N, C_in, C_out, H, W,
                                      spec.k, spec.T, spec.delta, spec.decay_conv, spec.th_conv, out_layout,
                                      _ptr(out), C.c_void_p(_stream(stream))), "vdt_dvs_conv_bucketed")
    return out


def dense_supported(C_in, k):
    """vdt_dvs_conv_dense handles the layer (K*K*C_in <= 1152, K*K <= 32)."""
    return k * k <= 32 and k * k * C_in <= 1152


def conv_dense(x, w_hwio, N, C_in, C_out, H, W, spec, in_layout=LAYOUT_NCHW, out_layout=LAYOUT_NCHW,
               stream=None):
    """k_bucketize_conv + conv_bucketed_early in one launch, straight from the
    input spike map x (same results as bucketize_sites + conv_bucketed)."""
    import torch
    out = torch.empty((N * C_out * H * W,), dtype=torch.float32, device=x.device)
    check(lib().vdt_dvs_conv_dense(_ptr(x), in_layout, _ptr(w_hwio), N, C_in, C_out, H, W, spec.k, spec.T,
                                   spec.delta, spec.decay_conv, spec.th_conv, out_layout, _ptr(out),
                                   C.c_void_p(_stream(stream))), "vdt_dvs_conv_dense")
    return out


def conv_layer(x, w_hwio, N, C_in, C_out, H, W, spec, stream=None):
    """A bucketed CuLIF conv layer on an NCHW map: the fused kernel where it
    applies, else bucketize_sites + conv_bucketed."""
    if dense_supported(C_in, spec.k):
        return conv_dense(x, w_hwio, N, C_in, C_out, H, W, spec, stream=stream)
    return conv_bucketed(bucketize_sites(x, N, C_in, H, W, spec, stream), w_hwio, N, C_in, C_out, H, W, spec,
                         stream=stream)


def pool(x, N, Cc, H, W, spec, layout=LAYOUT_NCHW, stream=None):
    import torch
    out = torch.empty((N * Cc * (H // 2) * (W // 2),), dtype=torch.float32, device=x.device)
    check(lib().vdt_dvs_pool(_ptr(x), _ptr(out), N, Cc, H, W, layout, spec.T, spec.delta, spec.decay_conv,
                             spec.th_conv, C.c_void_p(_stream(stream))), "vdt_dvs_pool")
    return out


def fc1_recurrent(buckets, w_t, rec_t, N, F_in, F_out, spec, stream=None, workspace=True):
    """fc1_bucketed_recurrent.  workspace=True hands the feed-forward sums'
    scratch over from torch's caching allocator (vdt_dvs_fc1_recurrent_ws);
    False lets the library allocate it stream-ordered per call."""
    import torch
    off, cin, tin = buckets
    out = torch.empty((N * F_out,), dtype=torch.float32, device=off.device)
    args = (_ptr(off), _ptr(cin), _ptr(tin), _ptr(w_t), _ptr(rec_t), N, F_in, F_out,
            spec.T, spec.delta, spec.decay_fc, spec.th_fc, _ptr(out))
    if workspace:
        nbytes = lib().vdt_dvs_fc1_scratch_bytes(N, F_out, spec.T, spec.delta)
        ws = torch.empty((max(nbytes, 4) // 4,), dtype=torch.float32, device=off.device)
        check(lib().vdt_dvs_fc1_recurrent_ws(*args, _ptr(ws), nbytes, C.c_void_p(_stream(stream))),
              "vdt_dvs_fc1_recurrent_ws")
    else:
        check(lib().vdt_dvs_fc1_recurrent(*args, C.c_void_p(_stream(stream))), "vdt_dvs_fc1_recurrent")
    return out


def fc2(buckets, w_t, N, F_in, F_out, spec, stream=None):
    import torch
    off, cin, tin = buckets
    out = torch.empty((N * F_out,), dtype=torch.float32, device=off.device)
    check(lib().vdt_dvs_fc2(_ptr(off), _ptr(cin), _ptr(tin), _ptr(w_t), N, F_in, F_out, spec.T, spec.delta,
                            spec.decay_fc, spec.th_fc, _ptr(out), C.c_void_p(_stream(stream))), "vdt_dvs_fc2")
    return out


def internal_spec(spec: nets.DvsSpec) -> nets.DvsSpec:
    """Chunk width the engine runs a network at.  Every stage's result is the
    same for any chunk width dividing T (each neuron sees the same per-step
    inputs in the same order; the scan ends at T), so when the configured
    width divides T the engine buckets at 8 (narrower per-chunk slot tables,
    four channels per lane); otherwise the configured width is kept, with the
    reference's scan past T in the last chunk."""
    if spec.T % spec.delta == 0 and spec.T % 8 == 0:
        return dataclasses.replace(spec, delta=8)
    return spec


def run(spec: nets.DvsSpec, w: DvsWeights, frames, keep=False, stream=None):
    """The reference main's per-batch sequence (t3:262-296) on the device:
    frames [N, C_in, H, W, T] -> maps, outputs [N, classes], predictions."""
    spec0, spec = spec, internal_spec(spec)
    N = frames.shape[0]
    s = spec.stage_shapes()
    c1n, c2n, c3n = spec.convs
    H, W = spec.H, spec.W
    maps = []
    x = conv1_raw(frames, w.conv1, spec0, stream)             # frame windows of the configured width
    maps.append(x)
    x = conv_layer(x, w.conv2, N, c1n, c2n, H, W, spec, stream)
    maps.append(x)
    x = pool(x, N, c2n, H, W, spec, stream=stream)
    maps.append(x)
    H2, W2 = H // 2, W // 2
    x = conv_layer(x, w.conv3, N, c2n, c3n, H2, W2, spec, stream)
    maps.append(x)
    x = pool(x, N, c3n, H2, W2, spec, stream=stream)
    maps.append(x)
    x = fc1_recurrent(bucketize_rows(x, N, s["fc1_in"], spec, stream), w.fc1_t, w.rec_t, N, s["fc1_in"],
                      spec.hidden, spec, stream)
    maps.append(x)
    x = fc2(bucketize_rows(x, N, spec.hidden, spec, stream), w.fc2_t, N, spec.hidden, spec.classes, spec, stream)
    maps.append(x)
    pred = readout(x, N, spec.classes, nets.READ_ARGMIN_LOWEST, stream=stream)
    res = {"out": x.reshape(N, spec.classes), "pred": pred}
    if keep:
        res["maps"] = maps
    return res


def run_host_batches(spec: nets.DvsSpec, w: DvsWeights, h_frames, outs=None, preds=None):
    """Several batches end to end from host memory, pipelined: batch i+1's
    frames are copied (a second device slot, a copy stream) while batch i
    runs on the current stream, and batch i's outputs are copied back while
    batch i+1 runs.  h_frames: pinned CPU tensors [N, C_in, H, W, T] of one
    shape; outs / preds: per batch, pinned tensors [N, classes] / [N]
    (allocated when None).  Same results as run() per batch; synchronous."""
    import torch
    n = len(h_frames)
    if n == 0:
        return [], []
    dev = w.conv1.device
    N = h_frames[0].shape[0]
    if outs is None:
        outs = [torch.empty((N, spec.classes), dtype=torch.float32).pin_memory() for _ in range(n)]
    if preds is None:
        preds = [torch.empty((N,), dtype=torch.int32).pin_memory() for _ in range(n)]
    if len(outs) != n or len(preds) != n:
        raise ValueError(f"{n} batches need {n} outputs and predictions, got {len(outs)} and {len(preds)}")
    comp = torch.cuda.current_stream(dev)
    copy = torch.cuda.Stream(dev)
    slots = [torch.empty(h_frames[0].shape, dtype=torch.float32, device=dev) for _ in range(min(2, n))]
    h2d = [torch.cuda.Event(), torch.cuda.Event()]
    done = [torch.cuda.Event(), torch.cuda.Event()]
    with torch.cuda.stream(copy):
        slots[0].copy_(h_frames[0], non_blocking=True)
        h2d[0].record(copy)
    for i in range(n):
        s = i & 1
        comp.wait_event(h2d[s])
        r = run(spec, w, slots[s])
        done[s].record(comp)
        if i + 1 < n:                                         # next frames, overlapping this batch
            s1 = (i + 1) & 1
            with torch.cuda.stream(copy):
                if i >= 1:
                    copy.wait_event(done[s1])                 # batch i - 1 left the slot
                slots[s1].copy_(h_frames[i + 1], non_blocking=True)
                h2d[s1].record(copy)
        with torch.cuda.stream(copy):
            copy.wait_event(done[s])
            outs[i].copy_(r["out"], non_blocking=True)
            preds[i].copy_(r["pred"], non_blocking=True)
        r["out"].record_stream(copy)                          # not reused before its copy ends
        r["pred"].record_stream(copy)
    copy.synchronize()
    comp.synchronize()
    return outs, preds

