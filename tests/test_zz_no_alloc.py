"""frc_run_device_fixed (hidden hand-off in the library's fixed device array,
no allocation in the call) against frc_run_device on the same inputs.

Collected last (file name) so it also runs after every other GPU test has
used the library; it passes alone too.  Tolerance: the per-token relative L2
bar of the parity tests (both calls run the same kernel, so in practice the
outputs are identical)."""
import numpy as np
import pytest

import fronk_b200 as fb
from oracle import OK, INVALID
from tests.helpers import make_layers, request, rel_l2

pytestmark = pytest.mark.gpu
SEED = 0x5EED
TOL = 1e-5


def _device(torch, arr):
    return torch.from_numpy(np.ascontiguousarray(arr)).cuda()


def test_fixed_scratch_matches_context_scratch(gpu):
    import torch
    hidden, layer = 2048, 3
    g = fb.geometry(hidden)
    cases = [request(hidden, 4, SEED + 91, 0.5), request(hidden, 3, SEED + 92, 0.0)]
    experts = np.concatenate([c[0].ravel() for c in cases])
    with fb.Context(0, hidden) as ctx:
        for b, arr in make_layers(g, SEED, list(range(20)), experts, shared=True).items():
            assert ctx.load_layer(b, layer, arr) == OK, ctx.last_error
        stream = torch.cuda.current_stream().cuda_stream
        for e, gate, x in cases:
            T = x.shape[0]
            de, dg, dx = _device(torch, e.astype(np.uint16)), _device(torch, gate), _device(torch, x)
            y_ctx = torch.full((T, hidden), np.nan, dtype=torch.float32, device="cuda")
            ctx.run_device(layer, T, de.data_ptr(), dg.data_ptr(), dx.data_ptr(), None, None, y_ctx.data_ptr(),
                           fb.ACT_Q8, 0, stream)
            assert ctx.status(stream) == OK, ctx.last_error
            ref = y_ctx.cpu().numpy()
            for _ in range(2):  # two calls in a row on the same fixed array
                y_fix = torch.full((T, hidden), np.nan, dtype=torch.float32, device="cuda")
                ctx.run_device_fixed(layer, T, de.data_ptr(), dg.data_ptr(), dx.data_ptr(), None, None,
                                     y_fix.data_ptr(), fb.ACT_Q8, 0, stream)
                assert ctx.status(stream) == OK, ctx.last_error
                out = y_fix.cpu().numpy()
                assert max(rel_l2(r, a) for r, a in zip(ref, out)) <= TOL


def test_fixed_scratch_rejects_oversize_call(gpu):
    import torch
    hidden, layer = 2048, 0
    g = fb.geometry(hidden)
    e, gate, x = request(hidden, 5, SEED + 93, 0.0)
    with fb.Context(0, hidden) as ctx:
        for b, arr in make_layers(g, SEED, list(range(20)), e, shared=True).items():
            assert ctx.load_layer(b, layer, arr) == OK, ctx.last_error
        de, dg, dx = _device(torch, e.astype(np.uint16)), _device(torch, gate), _device(torch, x)
        y = torch.zeros((5, hidden), dtype=torch.float32, device="cuda")
        before = ctx.launches
        with pytest.raises(fb.FrcError) as err:
            ctx.run_device_fixed(layer, 5, de.data_ptr(), dg.data_ptr(), dx.data_ptr(), None, None, y.data_ptr(),
                                 fb.ACT_Q8, 0, torch.cuda.current_stream().cuda_stream)
        assert err.value.code == INVALID and "fixed scratch" in ctx.last_error
        assert ctx.launches == before
        assert not bool(y.any())
