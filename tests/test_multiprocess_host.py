"""The in-box sharding on CPU: two gloo ranks own the planner's halves of the
slices, compute their gated partials (the oracle port of the GPU
arithmetic), and an all-reduce of the partials equals the whole layer.  The
same host logic drives the NCCL path of bench.py."""
import os
import socket

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, hidden, q):
    import sys
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist
    import fronk_b200 as fb
    from fronk_b200 import planner
    from oracle import Oracle, OK, Q4_K, MXFP4
    from tests.helpers import make_layers, request
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        oracle = Oracle()
        g = fb.geometry(hidden)
        e, gt, x = request(hidden, 3, 0x5EED + 5, 0.5)
        blocks = list(range(20))
        layers = make_layers(g, 0x5EED, blocks, e, shared=True)
        mine = planner.owned_blocks(rank, world)
        rc, y_part, _ = oracle.port_run(oracle.model(hidden, Q4_K, MXFP4, {b: layers[b] for b in mine}), e, gt, x)
        assert rc == OK
        t = torch.from_numpy(np.ascontiguousarray(y_part))
        dist.all_reduce(t)
        if rank == 0:
            rc, y_all, _ = oracle.port_run(oracle.model(hidden, Q4_K, MXFP4, layers), e, gt, x)
            assert rc == OK
            err = max(float(np.linalg.norm(a - b) / np.linalg.norm(a)) for a, b in zip(y_all, t.numpy()))
            q.put(("ok", err, mine))
        else:
            q.put(("ok", 0.0, mine))
    except Exception as exc:  # noqa: BLE001
        q.put(("error", repr(exc), None))
    finally:
        dist.destroy_process_group()


def test_two_rank_partials_sum_to_whole(built):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, 2048, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(r[0] == "ok" for r in results), results
    owned = sorted(r[2] for r in results)
    assert owned == [list(range(10)), list(range(10, 20))]
    err = max(r[1] for r in results)
    assert err <= 1e-6, err
