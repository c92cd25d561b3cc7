"""CPU checks of the expected outputs bench.py compares its timed steps with
(tests/golden/bench_parity.npz): the oracle reproduces them for the small
configurations, and bench.py's comparison flags a single changed value."""
import numpy as np

import bench_parity_helpers as H


def test_fixture_covers_every_bench_workload():
    g = H.load()
    for config in ("vgg16", "lenet5_b1024", "lenet5", "dvs", "dvs_ref"):
        B = int(g[f"{config}_batch"])
        assert g[f"{config}_pred"].shape == (B,)
        assert len(str(g[f"{config}_out_sha256"])) == 64


def test_oracle_reproduces_the_stored_outputs():
    import make_bench_parity as M
    g = H.load()
    for config in ("lenet5_b1024", "dvs_ref"):
        out, pred = M.expected(config)
        assert M.digest(out) == str(g[f"{config}_out_sha256"]), config
        assert np.array_equal(pred, g[f"{config}_pred"].astype(np.int32)), config


def test_bench_comparison_flags_one_changed_value():
    import bench
    import make_bench_parity as M
    out, pred = M.expected("lenet5_b1024")
    ok = bench.stored_parity("lenet5_b1024", out, pred, out.shape[0])
    assert ok["checked"] and ok["result"] == "bit-exact"
    bad = out.copy()
    bad[7, 3] = np.nextafter(bad[7, 3], np.float32(1e9))       # one ulp on one value
    r = bench.stored_parity("lenet5_b1024", bad, pred, out.shape[0])
    assert r["result"] == "MISMATCH" and not r["out_sha256_equal"] and r["pred_differing"] == 0
    p2 = pred.copy()
    p2[0] = (p2[0] + 1) % 10
    assert bench.stored_parity("lenet5_b1024", out, p2, out.shape[0])["pred_differing"] == 1
    assert not bench.stored_parity("lenet5_b1024", out, pred, 512)["checked"]     # other batch size
