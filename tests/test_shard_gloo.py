"""CPU multi-process tests of the N>1 path (world_size 2, gloo): batch
sharding + prediction gather give exactly the single-process result, and a
rank that fails is detected on the host by the survivors' bounded collective
timeout (no GPU involved)."""
import os
import sys
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import ROOT


def _setup(rank, world, port, timeout_s=30):
    import datetime

    import torch.distributed as dist
    sys.path.insert(0, os.path.join(ROOT, "vd-ttfs_b200"))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _worker_infer(rank, world, port, q):
    import torch
    dist = _setup(rank, world, port)
    import oracle as O
    from vdttfs import nets, shard, synth
    net = nets.lenet5()
    layers = synth.kaiming_layers(net, 1)
    img = synth.images(1, 37, 28, 28, 1, 0.8, stream=3)       # uneven split: 19 + 18

    def local(x):
        r = O.run_net(net, layers, O.encode_linear(x, net.T))
        return torch.from_numpy(r["out"]), torch.from_numpy(r["pred"])

    out, pred = shard.run_sharded(local, img, world, rank)
    if rank == 0:
        q.put((out.numpy(), pred.numpy()))
    dist.destroy_process_group()


def _free_port():
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_bounds_cover_batch():
    sys.path.insert(0, os.path.join(ROOT, "vd-ttfs_b200"))
    from vdttfs.shard import shard_bounds
    for total in (0, 1, 7, 256, 65536, 65537):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_bounds(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


def test_two_rank_gather_equals_single_process(O):
    from vdttfs import nets, synth
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker_infer, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    out, pred = q.get(timeout=120)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    net = nets.lenet5()
    img = synth.images(1, 37, 28, 28, 1, 0.8, stream=3)
    ref = O.run_net(net, synth.kaiming_layers(net, 1), O.encode_linear(img, net.T))
    assert np.array_equal(out.view(np.int32), ref["out"].view(np.int32))
    assert np.array_equal(pred, ref["pred"])


def _worker_fail(rank, world, port, q):
    import torch
    dist = _setup(rank, world, port, timeout_s=5)
    if rank == 1:
        raise SystemExit(3)                    # a rank that dies before its step
    t0 = time.time()
    try:
        dist.all_gather_into_tensor(torch.zeros(2 * 4, dtype=torch.int32), torch.zeros(4, dtype=torch.int32))
        q.put(("no-error", time.time() - t0))
    except Exception as e:                      # the survivor sees a bounded error
        q.put((type(e).__name__, time.time() - t0))


def test_failed_rank_is_detected_by_bounded_timeout():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker_fail, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    kind, dt = q.get(timeout=120)
    for p in ps:
        p.join(timeout=60)
    assert kind != "no-error"
    assert dt < 60
    assert ps[1].exitcode == 3
