"""Bursts above 16 tokens: the tensor-core prefill path (MXFP4 weights, Q8
activations) against the oracle's restatement of its arithmetic
(or_prefill_run), through the C ABI; and the bursts that run as 16-token
chunks of the decode kernel."""
import numpy as np
import pytest

import fronk_b200 as fb
from oracle import Oracle, MXFP4, Q4_K, OK, INVALID, NUMERIC
from tests.helpers import make_layers, request, rel_l2

pytestmark = pytest.mark.gpu
SEED = 0x5EED


@pytest.fixture(scope="module")
def oracle():
    return Oracle()


def _setup(ctx, oracle, blocks, e, hidden=2048, gate=MXFP4):
    g = fb.geometry(hidden, gate_type=gate, down_type=MXFP4)
    layers = make_layers(g, SEED, blocks, e, shared=True)
    for b, arr in layers.items():
        assert ctx.load_layer(b, 0, arr) == OK, ctx.last_error
    return oracle.model(hidden, gate, MXFP4, layers), layers


@pytest.mark.parametrize("tokens,blocks", [(17, [0]), (40, [0, 3, 7]), (100, [1, 2, 5, 6, 9, 19])])
def test_prefill_bitexact_with_oracle(gpu, oracle, tokens, blocks):
    """y, the int8 hidden values and their scales, bit for bit (the kernel and
    the oracle form the same exact block terms, sum them in double in the
    same order and round once), and y within 1e-5 of the reference's ref-q8."""
    e, gt, x = request(2048, tokens, SEED + tokens)
    with fb.Context(0, 2048, gate_type=MXFP4, down_type=MXFP4) as ctx:
        m, layers = _setup(ctx, oracle, blocks, e)
        rc, y = ctx.run(0, e, gt, x)
        assert rc == OK, ctx.last_error
        hq, hs = ctx.debug_prefill_hidden()
    rc, y_ref, hq_ref, hs_ref = oracle.prefill_run(m, e, gt, x, want_hidden=True)
    assert rc == OK
    assert np.array_equal(hq, hq_ref)
    assert np.array_equal(hs.view(np.uint32), hs_ref.view(np.uint32))
    assert max(rel_l2(y_ref[t], y[t]) for t in range(tokens)) <= 1e-5
    assert np.array_equal(y.view(np.uint32), y_ref.view(np.uint32))
    # the reference's ref-q8 (bit-identical restatement, 16 tokens a call;
    # a token's result depends only on its own row)
    for t0 in range(0, tokens, 16):
        sl = slice(t0, min(tokens, t0 + 16))
        rc, y_q8 = oracle.ref_run(m, e[sl], gt[sl], x[sl], 1)
        assert rc == OK
        errs = [rel_l2(r, a) for r, a in zip(y_q8, y[sl])]
        assert max(errs) <= 1e-5, ("vs ref-q8", errs)


@pytest.mark.parametrize("hidden,tokens,distinct", [(2560, 20, True), (2048, 300, False)])
def test_prefill_other_shapes(gpu, oracle, hidden, tokens, distinct):
    """The reference's own hidden size (d = 2560: ten 256-weight chunks, 20
    row tiles), and 300 tokens that all pick the same ten experts (five
    64-token tiles of each expert)."""
    e, gt, x = request(hidden, tokens, SEED + hidden + tokens, distinct=distinct)
    with fb.Context(0, hidden, gate_type=MXFP4, down_type=MXFP4) as ctx:
        m, layers = _setup(ctx, oracle, [5, 6, 12], e, hidden)
        rc, y = ctx.run(0, e, gt, x)
        assert rc == OK, ctx.last_error
        hq, hs = ctx.debug_prefill_hidden()
    rc, y_ref, hq_ref, hs_ref = oracle.prefill_run(m, e, gt, x, want_hidden=True)
    assert rc == OK
    assert np.array_equal(hq, hq_ref) and np.array_equal(hs.view(np.uint32), hs_ref.view(np.uint32))
    assert np.array_equal(y.view(np.uint32), y_ref.view(np.uint32))


@pytest.mark.parametrize("gate", [MXFP4, Q4_K])
def test_prefill_zipf_512_tokens_all_blocks(gpu, oracle, gate):
    """configs[4]'s shape: 512 tokens, Zipf(1.1) expert popularity, all 20
    blocks (device-filled units), on MXFP4 and on the reference's Q4_K
    gate/up rows.  Tokens are independent, so a sample of them is checked
    against the oracle bit for bit."""
    g = fb.geometry(2048, gate_type=gate, down_type=MXFP4)
    e, gt, x = fb.synth_request(2048, 512, SEED + 512, zipf=1.1)
    pool = np.concatenate([fb.synth_slice(g, SEED, i) for i in range(16)])
    sb = fb.slice_bytes(g)
    with fb.Context(0, 2048, gate_type=gate, down_type=MXFP4) as ctx:
        ctx.pool_load(pool, fb.synth_shared(g, SEED, 1 << 20))
        for b in range(20):
            ctx.fill_layer(b, 0, SEED)
        rc, y = ctx.run(0, e, gt, x)
        assert rc == OK, ctx.last_error
        rc2, y2 = ctx.run(0, e, gt, x)
        assert rc2 == OK and np.array_equal(y.view(np.uint32), y2.view(np.uint32))  # repeatable
    sample = [0, 1, 77, 255, 400, 511]
    layers = {}
    for b in range(20):
        arr = np.zeros(fb.layer_bytes(g), np.uint8)
        for ident in set(int(v) for v in e[sample].ravel()):
            k = fb.pool_pick(SEED, b, 0, ident, 16)
            arr[ident * sb:(ident + 1) * sb] = pool[k * sb:(k + 1) * sb]
        layers[b] = arr
    m = oracle.model(2048, gate, MXFP4, layers)
    rc, y_ref, _, _ = oracle.prefill_run(m, e[sample], gt[sample], x[sample])
    assert rc == OK
    assert np.array_equal(y[sample].view(np.uint32), y_ref.view(np.uint32))


@pytest.mark.parametrize("gate,tokens", [(MXFP4, 36), (Q4_K, 100)])
def test_prefill_with_the_shared_expert(gpu, oracle, gate, tokens):
    """A nonzero shared-expert gate keeps a long burst on the tensor-core path:
    the Q8_0 shared expert is expert 512 (its pairs after the routed ones,
    operands in natural order, each block's exact Z times d * 2^E, added
    after the token's routed experts).  hq, hscale and y bit for bit against
    the oracle, y within 1e-5 of ref-q8; a token without a shared gate skips
    it."""
    e, gt, x = request(2048, tokens, SEED + tokens + 7, shared_gate=0.3)
    gt[5, 10] = 0.0
    with fb.Context(0, 2048, gate_type=gate, down_type=MXFP4) as ctx:
        m, layers = _setup(ctx, oracle, [2, 4, 13], e, gate=gate)
        rc, y = ctx.run(0, e, gt, x)
        assert rc == OK, ctx.last_error
        hq, hs = ctx.debug_prefill_hidden()
    rc, y_ref, hq_ref, hs_ref = oracle.prefill_run(m, e, gt, x, want_hidden=True)
    assert rc == OK
    assert hq.shape[0] == tokens * 10 + tokens - 1
    assert np.array_equal(hq, hq_ref)
    assert np.array_equal(hs.view(np.uint32), hs_ref.view(np.uint32))
    assert np.array_equal(y.view(np.uint32), y_ref.view(np.uint32))
    for t0 in range(0, tokens, 16):
        sl = slice(t0, min(tokens, t0 + 16))
        rc, y_q8 = oracle.ref_run(m, e[sl], gt[sl], x[sl], 1)
        assert rc == OK
        assert max(rel_l2(r, a) for r, a in zip(y_q8, y[sl])) <= 1e-5


def test_prefill_shared_expert_nonfinite_scale_is_numeric(gpu, oracle):
    """An infinite fp16 scale in a block of the shared expert's Q8_0 down rows:
    NUMERIC whatever the gate, y untouched."""
    e, gt, x = request(2048, 20, SEED + 21, shared_gate=0.2)
    g = fb.geometry(2048, gate_type=MXFP4, down_type=MXFP4)
    bad = make_layers(g, SEED, [1], e, shared=True)[1]
    # reference layout of the shared slice: 64 gate/up rows of d/32 34-byte
    # Q8_0 blocks, then d down rows of one block; down row 77's fp16 scale
    off = 512 * fb.slice_bytes(g) + 2 * 32 * (2048 // 32) * 34 + 77 * 34
    bad[off:off + 2] = [0x00, 0x7c]
    sentinel = np.full(x.shape, 7.0, np.float32)
    with fb.Context(0, 2048, gate_type=MXFP4, down_type=MXFP4) as ctx:
        assert ctx.load_layer(1, 0, bad) == OK
        rc, y = ctx.run(0, e, gt, x, out=sentinel.copy())
        assert rc == NUMERIC and np.array_equal(y, sentinel)


def test_prefill_failures_leave_output_untouched(gpu, oracle):
    e, gt, x = request(2048, 24, SEED + 24)
    g = fb.geometry(2048, gate_type=MXFP4, down_type=MXFP4)
    sentinel = np.full(x.shape, 7.0, np.float32)
    bad = make_layers(g, SEED, [3], e, shared=True)[3]
    # E8M0 exponent 255: block 3 of up row 8 of a referenced slice (17-byte blocks, scale first)
    bad[int(e[5, 2]) * fb.slice_bytes(g) + 40 * fb.row_bytes(MXFP4, 2048) + 3 * 17] = 255
    with fb.Context(0, 2048, gate_type=MXFP4, down_type=MXFP4) as ctx:
        assert ctx.load_layer(3, 0, bad) == OK
        rc, y = ctx.run(0, e, gt, x, out=sentinel.copy())
        assert rc == NUMERIC and np.array_equal(y, sentinel)
        e2 = e.copy()
        e2[7, 3] = e2[7, 4]  # the same expert twice in one token
        rc, y = ctx.run(0, e2, gt, x, out=sentinel.copy())
        assert rc == INVALID and np.array_equal(y, sentinel)


def test_prefill_bf16_x_is_the_fp32_path_on_the_same_values(gpu, oracle):
    """configs[4]'s bf16 activations (FRC_RUN_X_BF16): the burst is widened
    exactly to fp32 on the device, so y equals the fp32 call on the widened
    values bit for bit (and the oracle); other calls with the flag are
    UNSUPPORTED and leave y alone."""
    import torch
    T = 64
    e, gt, x = request(2048, T, SEED + 640)
    xb = torch.from_numpy(x).to(torch.bfloat16)
    x_up = xb.float().numpy()
    dev = torch.device("cuda", 0)
    s = torch.cuda.current_stream().cuda_stream
    with fb.Context(0, 2048, gate_type=MXFP4, down_type=MXFP4) as ctx:
        m, layers = _setup(ctx, oracle, [0, 3, 11], e)
        rc, y32 = ctx.run(0, e, gt, x_up)
        assert rc == OK, ctx.last_error
        de = torch.from_numpy(e.astype(np.int16)).to(dev)
        dg = torch.from_numpy(gt).to(dev)
        dxb = xb.to(dev)
        dy = torch.zeros((T, 2048), device=dev)
        ctx.run_device(0, T, de.data_ptr(), dg.data_ptr(), dxb.data_ptr(), None, None, dy.data_ptr(), fb.ACT_Q8,
                       fb.RUN_X_BF16, s)
        torch.cuda.synchronize()
        assert ctx.status(s) == OK
        y16 = dy.cpu().numpy()
        assert np.array_equal(y16.view(np.uint32), y32.view(np.uint32))
        # a decode-sized call, and a burst with another flag: refused, y untouched
        sentinel = torch.full((T, 2048), 7.0, device=dev)
        for tokens, flags in ((8, fb.RUN_X_BF16), (T, fb.RUN_X_BF16 | fb.RUN_RMSNORM)):
            with pytest.raises(fb.FrcError) as err:
                ctx.run_device(0, tokens, de.data_ptr(), dg.data_ptr(), dxb.data_ptr(), None, None,
                               sentinel.data_ptr(), fb.ACT_Q8, flags, s)
            assert err.value.code == fb.UNSUPPORTED
        torch.cuda.synchronize()
        assert bool((sentinel == 7.0).all())
    rc, y_ref, _, _ = oracle.prefill_run(m, e, gt, x_up)
    assert rc == OK
    assert np.array_equal(y16.view(np.uint32), y_ref.view(np.uint32))


@pytest.mark.parametrize("hidden,tokens,blocks", [(2048, 17, [0]), (2048, 100, [1, 2, 5, 6, 9, 19]),
                                                  (2560, 40, [0, 3, 7])])
def test_prefill_q4k_gate_up_bitexact(gpu, oracle, hidden, tokens, blocks):
    """The reference's own unit layout (Q4_K gate/up, MXFP4 down) on the
    tensor-core path: Q4_K super-blocks staged by 3D tensor maps, nibbles as
    int8 operands, the exact per-group terms in double; hq, hscale and y bit
    for bit against the oracle, y within 1e-5 of ref-q8."""
    e, gt, x = request(hidden, tokens, SEED + 3 * tokens + hidden)
    with fb.Context(0, hidden, gate_type=Q4_K, down_type=MXFP4) as ctx:
        m, layers = _setup(ctx, oracle, blocks, e, hidden, gate=Q4_K)
        rc, y = ctx.run(0, e, gt, x)
        assert rc == OK, ctx.last_error
        hq, hs = ctx.debug_prefill_hidden()
    rc, y_ref, hq_ref, hs_ref = oracle.prefill_run(m, e, gt, x, want_hidden=True)
    assert rc == OK
    assert np.array_equal(hq, hq_ref)
    assert np.array_equal(hs.view(np.uint32), hs_ref.view(np.uint32))
    assert np.array_equal(y.view(np.uint32), y_ref.view(np.uint32))
    for t0 in range(0, tokens, 16):
        sl = slice(t0, min(tokens, t0 + 16))
        rc, y_q8 = oracle.ref_run(m, e[sl], gt[sl], x[sl], 1)
        assert rc == OK
        assert max(rel_l2(r, a) for r, a in zip(y_q8, y[sl])) <= 1e-5


def test_prefill_q4k_nonfinite_scale_is_numeric(gpu, oracle):
    """An infinite d in one super-block of a referenced Q4_K up row: NUMERIC,
    y untouched."""
    e, gt, x = request(2048, 24, SEED + 24)
    g = fb.geometry(2048, gate_type=Q4_K, down_type=MXFP4)
    bad = make_layers(g, SEED, [3], e, shared=True)[3]
    off = int(e[5, 2]) * fb.slice_bytes(g) + (32 + 8) * fb.row_bytes(Q4_K, 2048) + 3 * 144
    bad[off:off + 2] = [0x00, 0x7c]
    sentinel = np.full(x.shape, 7.0, np.float32)
    with fb.Context(0, 2048, gate_type=Q4_K, down_type=MXFP4) as ctx:
        assert ctx.load_layer(3, 0, bad) == OK
        rc, y = ctx.run(0, e, gt, x, out=sentinel.copy())
        assert rc == NUMERIC and np.array_equal(y, sentinel)
