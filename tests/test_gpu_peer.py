"""The in-box reduce over NVLink peer memory (FRC_RUN_PEER) on two GPUs:
each rank owns the planner's half of the slices, the kernels exchange their
partials through each other's inboxes, and y equals the whole layer (the
oracle port over all 20 slices, and the reference's ref-q8) on both ranks,
bit for bit the same on both.  The calls alternate one token (two CTAs an
SM) with sixteen (one CTA an SM), so row ownership changes from launch to
launch while the slots alternate by launch epoch.  Needs two GPUs; the IPC
handles go over a gloo group (host channel only).  The same calls through
the host-buffer entry point (frc_run_flags) give the same bits."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TOL = 1e-5


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    import sys
    sys.path.insert(0, ROOT)
    try:
        import torch
        import torch.distributed as dist
        import fronk_b200 as fb
        from fronk_b200 import planner
        from oracle import Oracle, OK, Q4_K, MXFP4
        from tests.helpers import make_layers, request
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        torch.cuda.set_device(rank)
        hidden, layer = 2048, 4
        g = fb.geometry(hidden)
        cases = [request(hidden, t, 0x5EED + 21 + i, 0.25 * (i % 3), True)
                 for i, t in enumerate((1, 16, 1, 1, 16, 3, 16, 16, 1, 2))]
        experts = np.concatenate([c[0].ravel() for c in cases])
        layers = make_layers(g, 0x5EED, list(range(20)), experts, shared=True)
        mine = planner.owned_blocks(rank, world)
        ys = []
        with fb.Context(rank, hidden) as ctx:
            for b in mine:
                assert ctx.load_layer(b, layer, layers[b]) == OK, ctx.last_error
            handles = [None] * world
            dist.all_gather_object(handles, ctx.peer_export(world))
            ctx.peer_attach(rank, world, handles)
            stream = torch.cuda.current_stream().cuda_stream
            for e, gate, x in cases:
                T = x.shape[0]
                de = torch.from_numpy(e.astype(np.uint16).view(np.int16)).cuda()
                dg, dx = torch.from_numpy(gate).cuda(), torch.from_numpy(x).cuda()
                y = torch.zeros((T, hidden), dtype=torch.float32, device="cuda")
                ctx.run_device(layer, T, de.data_ptr(), dg.data_ptr(), dx.data_ptr(), None, None, y.data_ptr(),
                               fb.ACT_Q8, fb.RUN_PEER, stream)
                assert ctx.status(stream) == OK, ctx.last_error
                ys.append(y.cpu().numpy())
            # the same calls from host buffers (frc_run_flags, FRC_RUN_PEER):
            # the same kernel and reduce, so the same bits
            for i, (e, gate, x) in enumerate(cases):
                rc, yh = ctx.run(layer, e, gate, x, flags=fb.RUN_PEER)
                assert rc == OK, ctx.last_error
                assert np.array_equal(yh.view(np.uint32), ys[i].view(np.uint32)), "host-buffer call differs"
            dist.barrier()
            ctx.peer_detach()
        gathered = [None] * world
        dist.all_gather_object(gathered, ys)
        if rank == 0:
            oracle = Oracle()
            m = oracle.model(hidden, Q4_K, MXFP4, layers)
            worst = 0.0
            for i, (e, gate, x) in enumerate(cases):
                rc, y_ref, _ = oracle.port_run(m, e, gate, x)
                rc2, y_q8 = oracle.ref_run(m, e, gate, x, 1)
                assert rc == OK and rc2 == OK
                assert np.array_equal(gathered[0][i].view(np.uint32), gathered[1][i].view(np.uint32)), "ranks differ"
                for ref in (y_ref, y_q8):
                    for r_, a_ in zip(ref, gathered[0][i]):
                        worst = max(worst, float(np.linalg.norm(r_ - a_) / np.linalg.norm(r_)))
            q.put(("ok", worst))
        else:
            q.put(("ok", 0.0))
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001
        q.put(("error", repr(exc)))


def test_peer_reduce_two_gpus(gpu):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(r[0] == "ok" for r in results), results
    assert max(r[1] for r in results) <= TOL, results
