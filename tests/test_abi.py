"""CPU checks of the C ABI: the library loads, exports every function that
include/vdttfs.h declares, and rejects bad input before touching a GPU."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from conftest import ROOT


def _declared():
    src = open(os.path.join(ROOT, "include", "vdttfs.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(vdt_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_the_boundary():
    names = _declared()
    for must in ["vdt_model_load_blob", "vdt_ctx_create", "vdt_infer", "vdt_infer_host",
                 "vdt_build_luts", "vdt_bucketize", "vdt_conv_bucketed", "vdt_layer_vmem",
                 "vdt_pool_min", "vdt_encode", "vdt_readout", "vdt_strerror"]:
        assert must in names


def test_library_exports_every_declared_symbol():
    from vdttfs import _lib
    L = _lib.lib()
    for name in _declared():
        assert hasattr(L, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_ctypes_signatures_match_the_header():
    """Every ctypes signature has as many arguments as the header declares."""
    from vdttfs import _lib
    src = open(os.path.join(ROOT, "include", "vdttfs.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    for m in re.finditer(r"\b(vdt_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", src, flags=re.S):
        name, params = m.group(1), " ".join(m.group(2).split())
        n = 0 if params in ("", "void") else params.count(",") + 1
        assert len(_lib.SIGNATURES[name][1]) == n, f"{name}: header has {n} parameters"


def test_status_strings_and_version():
    from vdttfs import _lib
    L = _lib.lib()
    assert b"sm_100a" in L.vdt_version()
    for s in range(7):
        assert L.vdt_strerror(s)


def _load(blob, net=None, cfg=None):
    from vdttfs import _lib, engine as E, nets
    net = net or nets.lenet5()
    descs = (_lib.LayerDesc * len(net.layers))(
        *[_lib.LayerDesc(l.kind, l.k, l.pad, int(l.pool_after), l.out) for l in net.layers])
    nd = _lib.NetDesc(net.in_h, net.in_w, net.in_c, net.tc_in, net.td_in, net.encoder, net.readout)
    cfg = cfg or E.time_cfg(net)
    h = C.c_void_p()
    st = _lib.lib().vdt_model_load_blob(blob, len(blob), descs, len(net.layers), C.byref(nd),
                                        C.byref(cfg), 0, C.byref(h))
    return st, _lib.lib().vdt_last_error().decode()


def test_blob_validation_happens_before_any_gpu_work():
    from vdttfs import blob, nets, synth
    net = nets.lenet5()
    good = blob.write_blob(synth.kaiming_layers(net, 1))
    assert _load(good[:-3])[0] == 2                      # truncated
    assert _load(good + b"\0\0\0\0")[0] == 2             # trailing bytes
    bad = bytearray(good)
    bad[0:4] = (7).to_bytes(4, "little")                  # wrong layer count
    assert _load(bytes(bad))[0] == 2
    bad = bytearray(good)
    bad[4:8] = (3).to_bytes(4, "little")                  # kernel ndim 3
    assert _load(bytes(bad))[0] == 2
    # topology mismatch: the VGG descriptor against the LeNet blob
    st, msg = _load(good, net=nets.vgg16())
    assert st == 2 and "layers" in msg


def test_time_config_validation():
    from vdttfs import blob, engine as E, nets, synth
    net = nets.lenet5()
    good = blob.write_blob(synth.kaiming_layers(net, 1))
    assert _load(good, cfg=E.time_cfg_raw(80, 3))[0] in (1, 5)       # delta 3: no kernel
    assert _load(good, cfg=E.time_cfg_raw(80, 16, lut_mode=1, decay_len=80))[0] == 1
    assert _load(good, cfg=E.time_cfg_raw(0, 16))[0] == 1


def test_per_stage_entry_points_reject_bad_arguments():
    from vdttfs import _lib, engine as E
    L = _lib.lib()
    cfg = E.time_cfg_raw(80, 8, 40.0)
    assert L.vdt_bucketize(None, 10, 4, 0, 1, C.byref(cfg), 0, None, None, None, None) == 1
    assert L.vdt_readout(None, 1, 10, 0, 9999.0, None, None) == 1
    assert L.vdt_pool_min(None, None, 1, 1, 1, 1, 9999.0, None) == 1
    assert L.vdt_infer(None, None, 0, 1, None, None) == 1


def test_dvs_flat_blob_validation_happens_before_any_gpu_work():
    """vdt_model_load_dvs_flat checks the descriptor and the blob's length
    before it touches a device: the reference-shaped blob holds the layers at
    the offsets of dvsgesture_weights_meta.txt (FC2 at float 1,287,296)."""
    from vdttfs import _lib, assets, dvs, nets, synth
    spec = nets.dvs_ref()
    layout, total = assets.dvs_flat_layout(spec)
    assert [off for _, _, off in layout] == [0, 1152, 74880, 222336, 238720, 1287296]
    blob = assets.write_dvs_flat(synth.dvs_weights(spec, 4), spec)
    assert len(blob) == 4 * total
    L = _lib.lib()
    h = C.c_void_p()

    def load(b, **over):
        d = dvs.dvs_desc(spec)
        for k, v in over.items():
            setattr(d, k, v)
        return L.vdt_model_load_dvs_flat(b, len(b), C.byref(d), 0, C.byref(h))

    assert load(blob[:-4]) == 2                           # one float short
    assert load(blob, H=30) == 1                          # two pools need H % 4 == 0
    assert load(blob, k=2) == 1                           # even kernel
    assert load(blob, T=0) == 1
    assert load(blob, delta=7) == 5                       # conv1 frame windows: delta 8, 16 or 32
    assert load(blob, hidden=100) == 5                    # recurrent FC1 width: multiple of 32
    assert L.vdt_model_load_dvs_flat(blob, len(blob), None, 0, C.byref(h)) == 1
    assert h.value is None
