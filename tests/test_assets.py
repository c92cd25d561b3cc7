"""The asset loaders against the reference's file formats (CPU)."""
import os

import numpy as np

from vdttfs import assets, nets, synth


def test_dvs_flat_layout_matches_the_reference_offsets():
    # the float offsets task 3 hard-codes for its 2x32x32 network (t3:240)
    layout, total = assets.dvs_flat_layout(nets.dvs_ref())
    offs = {name: off for name, _, off in layout}
    assert offs == {"conv1": 0, "conv2": 1152, "conv3": 74880, "fc1_rec": 222336, "fc1": 238720,
                    "fc2": 1287296}
    assert total == 1287296 + 10 * 128


def test_dvs_flat_round_trip(tmp_path):
    spec = nets.dvs_ref()
    wts = synth.dvs_weights(spec, 4)
    blob = assets.write_dvs_flat(wts, spec)
    p = tmp_path / "w.bin"
    p.write_bytes(blob + np.zeros(3456, "<f4").tobytes())      # a longer file: tail ignored
    back = assets.load_dvs_flat(str(p), spec)
    for k, v in wts.items():
        assert np.array_equal(back[k], v), k
    try:
        assets.load_dvs_flat(blob[:-4], spec)
        raise AssertionError("short blob accepted")
    except ValueError:
        pass


def test_image_sets_and_onehot_labels(tmp_path):
    rng = np.random.default_rng(0)
    imgs = rng.random((5, 32, 32, 3), dtype=np.float32)
    for i in range(5):
        imgs[i].astype("<f4").tofile(tmp_path / f"{i}.bin")
    labels = rng.integers(0, 10, 5)
    np.eye(10, dtype="<f4")[labels].tofile(tmp_path / "label_onehot")
    got = assets.load_images(str(tmp_path), 5, (32, 32, 3))
    assert np.array_equal(got, imgs)
    assert np.array_equal(assets.load_onehot(str(tmp_path / "label_onehot"), 5), labels)


def test_dvs_frames_and_int_labels(tmp_path):
    spec = nets.dvs_ref()
    fr = synth.dvs_frames(4, 2, spec)
    fr.astype("<f4").tofile(tmp_path / "train_data.bin")
    lab = np.array([3, 7])
    np.eye(spec.classes, dtype="<i4")[lab].tofile(tmp_path / "train_labels.bin")
    assert np.array_equal(assets.load_dvs_frames(str(tmp_path / "train_data.bin"), 2, spec), fr)
    assert np.array_equal(assets.load_onehot(str(tmp_path / "train_labels.bin"), 2, spec.classes, "<i4"), lab)


def test_network_output_size_is_the_last_map_flattened():
    """n_classes: an FC last layer's outputs; a conv last layer's whole map,
    after its pool when it has one."""
    from vdttfs import nets
    assert nets.vgg16().n_classes == 10 and nets.lenet5().n_classes == 10
    c = nets._conv
    assert nets.NetSpec("a", 7, 9, 3, (c(3, 8, 3, nets.PAD_SAME),)).n_classes == 7 * 9 * 8
    assert nets.NetSpec("b", 7, 9, 3, (c(3, 8, 3, nets.PAD_SAME, True),)).n_classes == 3 * 4 * 8
    assert nets.NetSpec("c", 7, 9, 3, (c(3, 8, 3, nets.PAD_VALID),)).n_classes == 5 * 7 * 8
