"""vdt_conv_layer_noalloc (the allocation-free layer step) against the
allocating per-stage entry points vdt_bucketize + vdt_conv_bucketed and
against the CPU oracle's bucketize + conv_bucketed (the reference's
k_bucketize / k_conv_bucketed restated, oracle/oracle.py).

The file name sorts last so that the test also runs after every other test
in the same process; it passes alone in a fresh process too.  Tolerance:
none -- both GPU paths run the same bucketing and integrator kernels, and
all three use the same host-libm LUTs, so the first-spike times must agree
bit for bit.
"""
import ctypes as C

import numpy as np
import pytest

from helpers import INF, bits_equal, spike_map

pytestmark = pytest.mark.gpu

# (conv or fc layer, time config) pairs; stagger layers use the (T+1)-entry
# LUT indexed by the input time, the others the T-entry LUT indexed by chunk
LAYERS = [
    dict(B=2, H=16, W=16, C_in=64, C_out=128, K=3, pad=1, is_fc=0, T=80, delta=4, tfs=40.0,
         lut_mode=1, tb_mode=0, gain=1.3),
    dict(B=4, H=12, W=12, C_in=6, C_out=16, K=5, pad=0, is_fc=0, T=80, delta=16, tfs=0.0,
         lut_mode=0, tb_mode=1, gain=0.4),
    dict(B=8, H=1, W=1, C_in=512, C_out=512, K=1, pad=0, is_fc=1, T=80, delta=8, tfs=40.0,
         lut_mode=1, tb_mode=0, gain=1.1),
]


def _setup(case, seed):
    import torch
    import oracle as O
    from vdttfs import engine as E
    rng = np.random.default_rng(seed)
    B, H, W, Ci, Co, K = case["B"], case["H"], case["W"], case["C_in"], case["C_out"], case["K"]
    Ho = 1 if case["is_fc"] else H + 2 * case["pad"] - K + 1
    Wo = 1 if case["is_fc"] else W + 2 * case["pad"] - K + 1
    fan = Ci * K * K
    Wt = (rng.standard_normal((K * K * Ci, Co)) * case["gain"] * np.sqrt(2.0 / fan)).astype(np.float32)
    bias = (rng.standard_normal(Co) * 0.01).astype(np.float32)
    T = case["T"]
    cfg = E.time_cfg_raw(T, case["delta"], case["tfs"], case["lut_mode"])
    hd, hth = O.update_luts(T, cfg.decay_len, 34.75, 0.0, 34.75, 0.0)     # the reference's libm tables
    dev = torch.device("cuda:0")
    t = lambda a: torch.from_numpy(a).to(dev)
    hx = [spike_map(rng, (B, H, W, Ci), fire=0.4, T=T, edges=True) for _ in range(2)]
    return dict(Wt=t(Wt), bias=t(bias), ld=t(hd), lt=t(hth), cfg=cfg, Ho=Ho, Wo=Wo, xs=[t(x) for x in hx],
                hx=hx, hW=Wt, hb=bias, hd=hd, hth=hth)


def _oracle(case, s, hx):
    import oracle as O
    B, H, W, Ci = case["B"], case["H"], case["W"], case["C_in"]
    n_cols = B if case["is_fc"] else B * H * W
    cfg = s["cfg"]
    off, cin, tin, _ = O.bucketize(hx, n_cols, Ci, cfg.T, cfg.delta, cfg.fire_start, case["tb_mode"])
    out, _ = O.conv_bucketed(off, cin, tin, s["hW"], s["hb"], s["hd"], s["hth"], 0, B, H, W, Ci, s["Ho"], s["Wo"],
                             case["C_out"], case["K"], case["pad"], case["is_fc"], cfg.T, cfg.delta,
                             cfg.fire_start, cfg.lut_mode)
    return out


def _allocating(case, s, x):
    from vdttfs import engine as E
    B, H, W, Ci = case["B"], case["H"], case["W"], case["C_in"]
    n_cols = B if case["is_fc"] else B * H * W
    off, cin, tin = E.bucketize(x, n_cols, Ci, s["cfg"], tb_mode=case["tb_mode"])
    return E.conv_bucketed(off, cin, tin, s["Wt"], s["bias"], s["ld"], s["lt"], 0, B, H, W, Ci,
                           s["Ho"], s["Wo"], case["C_out"], case["K"], case["pad"],
                           case["is_fc"], s["cfg"])


def _noalloc(case, s, x, out):
    from vdttfs._lib import lib
    ptr = lambda a: C.c_void_p(a.data_ptr())
    return lib().vdt_conv_layer_noalloc(
        ptr(x), case["tb_mode"], ptr(s["Wt"]), ptr(s["bias"]), ptr(s["ld"]), ptr(s["lt"]), 0,
        case["B"], case["H"], case["W"], case["C_in"], s["Ho"], s["Wo"], case["C_out"],
        case["K"], case["pad"], case["is_fc"], C.byref(s["cfg"]), ptr(out), C.c_void_p(0))


@pytest.mark.parametrize("case", LAYERS, ids=["conv_stagger", "conv_lenet", "fc"])
def test_noalloc_matches_allocating_entry_points_and_oracle_twice(case):
    import torch
    from vdttfs._lib import VDT_OK
    s = _setup(case, seed=17 + case["C_out"])
    n_out = case["B"] * s["Ho"] * s["Wo"] * case["C_out"]
    # two calls in a row on different inputs: the second must not see the first's lists
    for x, hx in zip(s["xs"], s["hx"]):
        out = torch.full((n_out,), -1.0, dtype=torch.float32, device=x.device)
        assert _noalloc(case, s, x, out) == VDT_OK
        ref = _allocating(case, s, x)
        torch.cuda.synchronize()
        a, b = out.cpu().numpy(), ref.cpu().numpy()
        assert bits_equal(a, b), f"{np.sum(a != b)} of {b.size} spike times differ from the allocating path"
        c = _oracle(case, s, hx)
        assert bits_equal(a, c), f"{np.sum(a != c)} of {c.size} spike times differ from the oracle"
        assert not (a == -1.0).any(), "every output neuron is written"
        assert 0.0 < np.mean(c < INF) < 1.0


def test_noalloc_rejects_a_layer_above_the_scratch_size():
    import torch
    from vdttfs._lib import lib
    limit = lib().vdt_noalloc_scratch_bytes()
    # a 224x224x64 batch of 8 needs ~240 MB of lists
    case = dict(LAYERS[0], B=8, H=224, W=224)
    n_cols, nc = 8 * 224 * 224, (80 + 3) // 4
    assert n_cols * (nc + 1) * 4 + 2 * n_cols * 64 * 4 > limit
    s = _setup(dict(LAYERS[0]), seed=3)
    x = torch.full((8 * 224 * 224 * 64,), 5.0, dtype=torch.float32, device="cuda:0")
    out = torch.full((8 * 224 * 224 * 128,), -1.0, dtype=torch.float32, device="cuda:0")
    s.update(Ho=224, Wo=224)
    assert _noalloc(case, s, x, out) == 6  # VDT_ERR_CAPACITY
    torch.cuda.synchronize()
    assert bool((out == -1.0).all()), "a rejected call must launch nothing"
