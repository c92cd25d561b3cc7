"""Python mirror of the engine's C ABI (include/vdttfs.h).

Names follow the reference's host helpers and kernels so a caller of the
reference program finds the same operations:

=========================  ==========================================  ==================================
here                       reference                                   C ABI
=========================  ==========================================  ==================================
Model(net, layers)         load_weights + per-layer update_LUTs        vdt_model_load_blob
Context.infer / infer_host the per-batch body of main                  vdt_infer / vdt_infer_host
update_LUTs                update_LUTs (t1:208, t2:236)                vdt_build_luts
encode_image               k_encode_image (t1:32, t2:32)               vdt_encode
bucketize                  k_bucketize (t1:45, t2:45), t3:70/93        vdt_bucketize
conv_bucketed              k_conv_bucketed (t1:83, t2:84)              vdt_conv_bucketed
layer_vmem                 k_layer_vmem (t2:172)                       vdt_layer_vmem
pooling                    k_pooling (t1:164, t2:192)                  vdt_pool_min
readout                    host argmin/argmax (t1:313, t2:391, t3:295) vdt_readout
=========================  ==========================================  ==================================

(t1/t2/t3 = the task 1/2/3 vdttfs_cuda programs of the reference.)
Device tensors are torch CUDA tensors; torch provides memory and streams only.
"""
from __future__ import annotations

import ctypes as C
import weakref

import numpy as np

from . import nets
from ._lib import LayerDesc, NetDesc, TimeCfg, VdtError, check, lib
from .blob import BlobLayer, write_blob

LUT_DEVICE, LUT_HOST_LIBM = 0, 1
LAYOUT_NHWC, LAYOUT_NCHW = 0, 1
TB_FLOOR_STAGGER, TB_TRUNC = 0, 1
KERNEL_CHUNK, KERNEL_SORTED, KERNEL_DENSE, KERNEL_VMEM, KERNEL_THREAD = 0, 1, 2, 3, 4
KERNEL_NAMES = {0: "k_integrate", 1: "k_sorted", 2: "k_dense", 3: "k_layer_vmem", 4: "k_thread"}


def _ptr(t) -> int:
    return 0 if t is None else int(t.data_ptr())


def _stream(stream) -> int:
    if stream is None:
        import torch
        return int(torch.cuda.current_stream().cuda_stream)
    return int(stream)


def time_cfg(net: nets.NetSpec, lut_source: int = LUT_DEVICE) -> TimeCfg:
    return TimeCfg(net.T, net.delta, net.tfs, net.vth_init, net.inf_time, net.lut_mode,
                   net.decay_len, lut_source)


def time_cfg_raw(T: int, delta: int, tfs: float = 0.0, lut_mode: int = nets.LUT_BY_TB,
                 decay_len: int | None = None, vth: float = 1.0, inf_time: float = 9999.0,
                 lut_source: int = LUT_DEVICE) -> TimeCfg:
    if decay_len is None:
        decay_len = T + 1 if lut_mode == nets.LUT_BY_TIN else T
    return TimeCfg(T, delta, tfs, vth, inf_time, lut_mode, decay_len, lut_source)


class Model:
    """An immutable loaded network (weights + LUTs on one device)."""

    def __init__(self, net: nets.NetSpec, layers, device: int = 0, lut_source: int = LUT_DEVICE):
        self.net = net
        blob = layers if isinstance(layers, (bytes, bytearray)) else write_blob(layers)
        self._blob = bytes(blob)
        descs = (LayerDesc * len(net.layers))(
            *[LayerDesc(l.kind, l.k, l.pad, int(l.pool_after), l.out) for l in net.layers])
        nd = NetDesc(net.in_h, net.in_w, net.in_c, net.tc_in, net.td_in, net.encoder, net.readout)
        self.cfg = time_cfg(net, lut_source)
        h = C.c_void_p()
        check(lib().vdt_model_load_blob(self._blob, len(self._blob), descs, len(net.layers),
                                        C.byref(nd), C.byref(self.cfg), device, C.byref(h)),
              "vdt_model_load_blob")
        self.h = h
        self.device = device
        nl, nc, wb = C.c_int(), C.c_int(), C.c_size_t()
        check(lib().vdt_model_info(h, C.byref(nl), C.byref(nc), C.byref(wb)), "vdt_model_info")
        self.n_classes = nc.value
        self.weight_bytes = wb.value
        self._contexts = weakref.WeakSet()   # closed before the model goes

    def luts(self, layer: int):
        d = np.zeros(self.net.decay_len, np.float32)
        th = np.zeros(self.net.T, np.float32)
        check(lib().vdt_model_luts(self.h, layer, d.ctypes.data, th.ctypes.data), "vdt_model_luts")
        return d, th

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


class Context:
    """Per-stream workspace for batches up to max_batch."""

    def __init__(self, model: Model, max_batch: int, stream=None, graphs: bool = True):
        self.model = model
        self.max_batch = max_batch
        self.stream = _stream(stream)
        h = C.c_void_p()
        check(lib().vdt_ctx_create(model.h, max_batch, C.c_void_p(self.stream), C.byref(h)),
              "vdt_ctx_create")
        self.h = h
        model._contexts.add(self)
        self.set_graphs(graphs)

    def set_graphs(self, on: bool):
        check(lib().vdt_ctx_set_graphs(self.h, int(on)), "vdt_ctx_set_graphs")

    def set_sub_batches(self, n: int):
        """1 or 2: run each batch as n halves on n streams (same results)."""
        check(lib().vdt_ctx_set_sub_batches(self.h, int(n)), "vdt_ctx_set_sub_batches")

    def set_counting(self, on: bool):
        check(lib().vdt_ctx_set_counting(self.h, int(on)), "vdt_ctx_set_counting")

    def counters(self):
        e, f = C.c_ulonglong(), C.c_ulonglong()
        check(lib().vdt_ctx_counters(self.h, C.byref(e), C.byref(f)), "vdt_ctx_counters")
        return e.value, f.value

    def layer_counters(self):
        """Per layer (events kept by its bucketing, synapses its integrator
        fetched) since the last read of either counter call."""
        n = len(self.model.net.layers)
        e, f = np.zeros(n, np.uint64), np.zeros(n, np.uint64)
        check(lib().vdt_ctx_layer_counters(self.h, n, e.ctypes.data, f.ctypes.data), "vdt_ctx_layer_counters")
        return [int(v) for v in e], [int(v) for v in f]

    def set_profiling(self, on: bool):
        check(lib().vdt_ctx_set_profiling(self.h, int(on)), "vdt_ctx_set_profiling")

    def layer_times(self):
        """Per-layer (bucketize, integrate, pool) milliseconds accumulated since
        the last call, and the number of batches they cover."""
        n = len(self.model.net.layers)
        a, b, c = (np.zeros(n, np.float32) for _ in range(3))
        nb = C.c_int()
        check(lib().vdt_ctx_layer_times(self.h, n, a.ctypes.data, b.ctypes.data, c.ctypes.data,
                                        C.byref(nb)), "vdt_ctx_layer_times")
        return a, b, c, nb.value

    def layer_kernels(self):
        """Integrator per layer: KERNEL_CHUNK, KERNEL_SORTED, KERNEL_DENSE,
        KERNEL_THREAD or KERNEL_VMEM (dense and thread layers launch no
        bucketize pass)."""
        n = len(self.model.net.layers)
        k = np.zeros(n, np.int32)
        check(lib().vdt_ctx_layer_kernels(self.h, n, k.ctypes.data), "vdt_ctx_layer_kernels")
        return [int(v) for v in k]

    def set_layer_kernel(self, layer: int, kernel: int):
        """Force one layer's integrator (KERNEL_*), or -1 for the automatic choice."""
        check(lib().vdt_ctx_set_layer_kernel(self.h, layer, kernel), "vdt_ctx_set_layer_kernel")

    def infer(self, x, pixels: bool = False, out=None, pred=None):
        """x: CUDA tensor [B, H, W, C] (spike times, or pixels if `pixels`)."""
        import torch
        B = x.shape[0]
        if out is None:
            out = torch.empty((B, self.model.n_classes), dtype=torch.float32, device=x.device)
        if pred is None:
            pred = torch.empty((B,), dtype=torch.int32, device=x.device)
        check(lib().vdt_infer(self.h, _ptr(x), int(pixels), B, _ptr(out), _ptr(pred)), "vdt_infer")
        return out, pred

    def infer_host(self, x: np.ndarray, pixels: bool = False, out=None, pred=None):
        """End to end from host memory (numpy or pinned torch CPU tensors)."""
        B = x.shape[0]
        if out is None:
            out = np.empty((B, self.model.n_classes), np.float32)
        if pred is None:
            pred = np.empty((B,), np.int32)

        def hp(a):
            return a.ctypes.data if isinstance(a, np.ndarray) else a.data_ptr()
        check(lib().vdt_infer_host(self.h, hp(x), int(pixels), B, hp(out), hp(pred)), "vdt_infer_host")
        return out, pred

    def infer_host_batches(self, xs, pixels: bool = False, outs=None, preds=None):
        """Several batches end to end from host memory, pipelined
        (vdt_infer_host_batches: the next batch's H2D copy overlaps this
        batch's compute).  xs: host arrays / pinned CPU tensors, all of one
        batch size; outs / preds: per batch, allocated when None."""
        n = len(xs)
        if n == 0:
            return [], []
        B = xs[0].shape[0]
        if any(x.shape[0] != B for x in xs):
            raise ValueError("every batch must have the same size")
        if outs is None:
            outs = [np.empty((B, self.model.n_classes), np.float32) for _ in range(n)]
        if preds is None:
            preds = [np.empty((B,), np.int32) for _ in range(n)]
        if len(outs) != n or len(preds) != n:
            raise ValueError(f"{n} batches need {n} outputs and predictions, got {len(outs)} and {len(preds)}")

        def hp(a):
            return a.ctypes.data if isinstance(a, np.ndarray) else a.data_ptr()
        arr = lambda items: (C.c_void_p * n)(*[hp(a) for a in items])
        check(lib().vdt_infer_host_batches(self.h, n, arr(xs), int(pixels), B, arr(outs), arr(preds)),
              "vdt_infer_host_batches")
        return outs, preds

    def trace(self, x, pixels: bool = False):
        """Whole network, returning every layer's output map (before pooling)."""
        import torch
        B = x.shape[0]
        maps = []
        for (_, _, _, ho, wo, co) in self.model.net.shapes():
            maps.append(torch.empty((B, ho, wo, co), dtype=torch.float32, device=x.device))
        arr = (C.c_void_p * len(maps))(*[_ptr(m) for m in maps])
        out = torch.empty((B, self.model.n_classes), dtype=torch.float32, device=x.device)
        pred = torch.empty((B,), dtype=torch.int32, device=x.device)
        check(lib().vdt_infer_trace(self.h, _ptr(x), int(pixels), B, arr, _ptr(out), _ptr(pred)),
              "vdt_infer_trace")
        return maps, out, pred

    def close(self):
        if self.h:
            lib().vdt_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------- per stage --
def update_LUTs(T, decay_len, tc_integ, td_integ, tc_fire, td_fire, vth_init=1.0, stream=None):
    import torch
    d = torch.empty(decay_len, dtype=torch.float32, device="cuda")
    th = torch.empty(T, dtype=torch.float32, device="cuda")
    check(lib().vdt_build_luts(T, decay_len, tc_integ, td_integ, tc_fire, td_fire, vth_init,
                               _ptr(d), _ptr(th), C.c_void_p(_stream(stream))), "vdt_build_luts")
    return d, th


def encode_image(px, encoder, tc=0.0, td=0.0, T=80, inf_time=9999.0, stream=None):
    import torch
    out = torch.empty_like(px)
    check(lib().vdt_encode(_ptr(px), _ptr(out), px.numel(), encoder, tc, td, T, inf_time,
                           C.c_void_p(_stream(stream))), "vdt_encode")
    return out


def bucketize(x, n_cols, c_in, cfg: TimeCfg, layout=LAYOUT_NHWC, hw=1, tb_mode=TB_FLOOR_STAGGER,
              stream=None):
    import torch
    nc = (cfg.T + cfg.delta - 1) // cfg.delta
    off = torch.zeros((n_cols, nc + 1), dtype=torch.int32, device=x.device)
    cin = torch.zeros((n_cols, c_in), dtype=torch.int32, device=x.device)
    tin = torch.zeros((n_cols, c_in), dtype=torch.float32, device=x.device)
    check(lib().vdt_bucketize(_ptr(x), n_cols, c_in, layout, hw, C.byref(cfg), tb_mode,
                              _ptr(off), _ptr(cin), _ptr(tin), C.c_void_p(_stream(stream))),
          "vdt_bucketize")
    return off, cin, tin


def conv_bucketed(off, cin, tin, kernel, bias, lut_decay, lut_th, t_min, B, H_in, W_in, C_in,
                  H_out, W_out, C_out, K, pad, is_fc, cfg: TimeCfg, stream=None):
    import torch
    out = torch.empty((B * H_out * W_out * C_out,), dtype=torch.float32, device=off.device)
    check(lib().vdt_conv_bucketed(_ptr(off), _ptr(cin), _ptr(tin), _ptr(kernel), _ptr(bias),
                                  _ptr(lut_decay), _ptr(lut_th), t_min, B, H_in, W_in, C_in,
                                  H_out, W_out, C_out, K, pad, int(is_fc), C.byref(cfg), _ptr(out),
                                  C.c_void_p(_stream(stream))), "vdt_conv_bucketed")
    return out


def layer_vmem(x, kernel, bias, lut_decay, B, C_in, C_out, cfg: TimeCfg, stream=None):
    import torch
    out = torch.empty((B * C_out,), dtype=torch.float32, device=x.device)
    check(lib().vdt_layer_vmem(_ptr(x), _ptr(kernel), _ptr(bias), _ptr(lut_decay), B, C_in, C_out,
                               C.byref(cfg), _ptr(out), C.c_void_p(_stream(stream))), "vdt_layer_vmem")
    return out


def pooling(x, B, H, W, Cc, inf_time=9999.0, stream=None):
    import torch
    out = torch.empty((B * (H // 2) * (W // 2) * Cc,), dtype=torch.float32, device=x.device)
    check(lib().vdt_pool_min(_ptr(x), _ptr(out), B, H, W, Cc, inf_time, C.c_void_p(_stream(stream))),
          "vdt_pool_min")
    return out


def readout(out, B, K, mode, inf_time=9999.0, stream=None):
    import torch
    pred = torch.empty((B,), dtype=torch.int32, device=out.device)
    check(lib().vdt_readout(_ptr(out), B, K, mode, inf_time, _ptr(pred), C.c_void_p(_stream(stream))),
          "vdt_readout")
    return pred


__all__ = ["Model", "Context", "update_LUTs", "encode_image", "bucketize", "conv_bucketed",
           "layer_vmem", "pooling", "readout", "time_cfg", "time_cfg_raw", "BlobLayer",
           "LUT_DEVICE", "LUT_HOST_LIBM"]
