"""The layer kernel's bounded waits on a GPU: a wait that runs out ends the
launch with an error status instead of hanging.  The grid barrier is made to
wait for arrivals that never come (frc_debug_barrier_extra) under a 1 ms limit
(frc_set_wait_limit): the call returns FRC_IO (frc_run) or frc_status reports
it (frc_run_device), y is left untouched, and the next call on the same
context is correct.  Nothing faults: every CTA gives up on its own clock."""
import time

import numpy as np
import pytest

import fronk_b200 as fb
from oracle import OK
from tests.helpers import make_layers, request, rel_l2

pytestmark = pytest.mark.gpu
SEED = 0x5EED


@pytest.mark.parametrize("tokens", [1, 16])
def test_barrier_wait_runs_out_and_context_recovers(gpu, oracle, tokens):
    hidden = 2048
    g = fb.geometry(hidden)
    e, gate, x = request(hidden, tokens, SEED + 90 + tokens, 0.5)
    with fb.Context(0, hidden) as ctx:
        layers = make_layers(g, SEED, [1, 6, 13], e, shared=True)
        for b, arr in layers.items():
            assert ctx.load_layer(b, 7, arr) == fb.OK, ctx.last_error
        rc, y_ok = ctx.run(7, e, gate, x, fb.ACT_Q8)
        assert rc == fb.OK, ctx.last_error
        ctx.set_wait_limit(1_000_000)
        ctx.debug_barrier_extra(1)
        sentinel = np.full((tokens, hidden), 7.0, np.float32)
        t0 = time.perf_counter()
        rc, y = ctx.run(7, e, gate, x, fb.ACT_Q8, out=sentinel.copy())
        dt = time.perf_counter() - t0
        assert rc == fb.IO, (rc, ctx.last_error)
        assert np.array_equal(y, sentinel), "output written on a failed call"
        assert dt < 1.0, dt
        # the device-pointer entry reports it through frc_status
        import torch
        dev = torch.device("cuda", 0)
        de = torch.from_numpy(e.astype(np.uint16).view(np.int16)).to(dev)
        dg, dx = torch.from_numpy(gate).to(dev), torch.from_numpy(x).to(dev)
        dy = torch.zeros((tokens, hidden), device=dev)
        s = torch.cuda.current_stream().cuda_stream
        ctx.run_device(7, tokens, de.data_ptr(), dg.data_ptr(), dx.data_ptr(), None, None, dy.data_ptr(), fb.ACT_Q8,
                       0, s)
        assert ctx.status(s) == fb.IO
        # back to normal: the same context computes the layer again, bit for bit
        ctx.debug_barrier_extra(0)
        rc, y2 = ctx.run(7, e, gate, x, fb.ACT_Q8)
        assert rc == fb.OK, ctx.last_error
        assert np.array_equal(y2.view(np.uint32), y_ok.view(np.uint32))
        ctx.run_device(7, tokens, de.data_ptr(), dg.data_ptr(), dx.data_ptr(), None, None, dy.data_ptr(), fb.ACT_Q8,
                       0, s)
        assert ctx.status(s) == fb.OK, ctx.last_error
        assert np.array_equal(dy.cpu().numpy().view(np.uint32), y_ok.view(np.uint32))
        ctx.set_wait_limit(2_000_000_000)
    rc, y_ref, _ = oracle.port_run(oracle.model(hidden, fb.Q4_K, fb.MXFP4, layers), e, gate, x)
    assert rc == OK and max(rel_l2(r, a) for r, a in zip(y_ref, y_ok)) <= 1e-5
