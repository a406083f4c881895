"""The one-token row-owner kernel (frc_layer_rb.cuh) against the item kernel
that serves larger bursts: the same values in the same order, so y and the
hidden activations must agree bit for bit, over slice counts 1..20, both
shared-expert cases, every routed layout, the reference geometry (d = 2560:
one CTA an SM), and consecutive overlapped launches (programmatic dependent
launch) on one stream.  Both are also checked against the oracle port and the
reference's ref-q8 (or_ref_run q8) within 1e-5."""
import numpy as np
import pytest

import fronk_b200 as fb
from oracle import OK, Q4_K, MXFP4, Q8_0
from tests.helpers import make_layers, request, rel_l2

pytestmark = pytest.mark.gpu
SEED = 0x5EED
TOL = 1e-5


@pytest.mark.parametrize("hidden,gt,dt", [(2048, Q4_K, MXFP4), (2560, Q4_K, MXFP4), (2048, MXFP4, Q8_0),
                                          (2048, Q8_0, MXFP4)])
def test_row_owner_equals_item_kernel(gpu, oracle, hidden, gt, dt):
    g = fb.geometry(hidden, 48, gt, dt)
    cases = [request(hidden, 1, SEED + 300 + i, sh, True) for i, sh in enumerate((0.0, 0.5, 0.0, 0.125))]
    experts = np.concatenate([c[0].ravel() for c in cases])
    for blocks in ([7], [0, 9, 19], list(range(20))):
        layers = make_layers(g, SEED + len(blocks), blocks, experts, shared=True)
        m = oracle.model(hidden, gt, dt, layers)
        with fb.Context(0, hidden, 48, gt, dt) as ctx:
            for b, arr in layers.items():
                assert ctx.load_layer(b, 3, arr) == OK, ctx.last_error
            for e, gate, x in cases:
                ctx.layer_variant(2)
                rc, y1 = ctx.run(3, e, gate, x, fb.ACT_Q8)
                assert rc == OK, ctx.last_error
                h1 = ctx.debug_hidden()
                ctx.layer_variant(0)
                rc, y0 = ctx.run(3, e, gate, x, fb.ACT_Q8)
                assert rc == OK, ctx.last_error
                h0 = ctx.debug_hidden()
                assert np.array_equal(h1.view(np.uint32), h0.view(np.uint32)), (len(blocks), "hidden")
                assert np.array_equal(y1.view(np.uint32), y0.view(np.uint32)), (len(blocks), "y")
                rc, y_ref, h_ref = oracle.port_run(m, e, gate, x, want_hidden=True)
                assert rc == OK and np.array_equal(h1.view(np.uint32), h_ref.view(np.uint32))
                assert rel_l2(y_ref[0], y1[0]) <= TOL
                rc, y_q8 = oracle.ref_run(m, e, gate, x, 1)
                assert rc == OK and rel_l2(y_q8[0], y1[0]) <= TOL, rel_l2(y_q8[0], y1[0])


def test_row_owner_overlapped_chain(gpu, oracle):
    """Eight overlapped launches on one stream (FRC_RUN_OVERLAP, the pass's
    form), each layer's input the previous output plus the residual, against
    the same chain run one synchronous launch at a time with the item kernel."""
    import torch
    hidden, L = 2048, 8
    g = fb.geometry(hidden)
    routes = [request(hidden, 1, SEED + 700 + l, 0.0) for l in range(L)]
    experts = np.concatenate([r[0].ravel() for r in routes])
    dev = torch.device("cuda", 0)
    outs = []
    for variant, flags in ((2, fb.RUN_RMSNORM | fb.RUN_OVERLAP), (0, fb.RUN_RMSNORM)):
        with fb.Context(0, hidden) as ctx:
            lay = make_layers(g, SEED, [1, 5, 12, 18], experts, shared=False)
            for l in range(L):
                for b, arr in lay.items():
                    assert ctx.load_layer(b, l, arr) == OK
            ctx.layer_variant(variant)
            ex = torch.from_numpy(np.stack([r[0] for r in routes]).astype(np.uint16).view(np.int16)).to(dev)
            gt = torch.from_numpy(np.stack([r[1] for r in routes])).to(dev)
            x0 = torch.from_numpy(routes[0][2]).to(dev)
            H = [torch.zeros((1, hidden), device=dev) for _ in range(2)]
            Y = [torch.zeros((1, hidden), device=dev) for _ in range(2)]
            s = torch.cuda.current_stream().cuda_stream
            for l in range(L):
                x = x0 if l <= 1 else H[(l - 1) % 2]
                x_add = None if l == 0 else Y[(l - 1) % 2].data_ptr()
                x_out = None if l == 0 else H[l % 2].data_ptr()
                ctx.run_device(l, 1, ex[l].data_ptr(), gt[l].data_ptr(), x.data_ptr(), x_add, x_out,
                               Y[l % 2].data_ptr(), fb.ACT_Q8, flags, s)
                if variant == 0:
                    assert ctx.status(s) == OK, ctx.last_error
            assert ctx.status(s) == OK, ctx.last_error
            outs.append(Y[(L - 1) % 2].cpu().numpy().copy())
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
