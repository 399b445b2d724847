"""sm_100a kernels vs the oracle, called through the C ABI (needs a B200)."""

import pytest
import torch

from helpers import seeded_w, seeded_x
from oracle import ops
from zimage_b200 import _lib

pytestmark = pytest.mark.gpu


def _act_quant(x, had=True, want_rot=True):
    M, K = x.shape
    xd = x.cuda().contiguous()
    q = torch.empty(M, K, dtype=torch.int8, device="cuda")
    sx = torch.empty(M, dtype=torch.bfloat16, device="cuda")
    xr = torch.empty(M, K, dtype=torch.bfloat16, device="cuda") if want_rot else None
    _lib.call("zib_act_quant", xd.data_ptr(), K, q.data_ptr(), K, sx.data_ptr(), _lib.ptr(xr), M, K,
              1 if had else 0, _lib.stream_of(xd))
    torch.cuda.synchronize()
    return q.cpu(), sx.cpu(), None if xr is None else xr.cpu()


@pytest.mark.parametrize("M,K", [(1, 128), (37, 3840), (256, 3840), (64, 10240), (5, 256)])
def test_act_quant_hadamard_bitexact(cuda, M, K):
    x = seeded_x(M, K, seed=M + K)
    if M > 3:
        x[2] = 0           # all-zero row: scale clamp path
        x[3] *= 1e4        # huge row
    q, sx, xr = _act_quant(x)
    oq, osx, oxr = ops.act_quant_had128(x)
    # the quantisation of the kernel's own rotation is exact reference arithmetic
    rq, rs = ops.quantize_rotated(xr)
    assert torch.equal(q, rq) and torch.equal(sx, rs.flatten())
    # the rotation itself matches the exact oracle except for rare fp32-sum roundings
    assert (xr != oxr).float().mean().item() <= 1e-5
    assert torch.equal(sx, osx.flatten())
    assert int((q != oq).sum()) == 0


def test_act_quant_vs_reference_matmul_rotation(cuda):
    """Against the reference's own bf16-matmul rotation (int8_linear.py:124-126)."""
    x = seeded_x(1024, 3840, seed=0)
    q, sx, _ = _act_quant(x, want_rot=False)
    rq, rsx, _ = ops.act_quant_had128_matmul(x)
    assert torch.equal(sx, rsx.flatten())
    assert (q != rq).float().mean().item() <= 1e-5
    assert int((q.int() - rq.int()).abs().max()) <= 1


def test_act_quant_midpoint_rows_bitexact(cuda):
    """Rows whose fp32 rotation products sit exactly on bf16 midpoints: the exact-residual
    rounding (int8_linear.py:124-126 rounds the exact product once) in the row kernels."""
    from helpers import midpoint_rows

    x, tie = midpoint_rows()
    assert int(tie.sum()) >= x.shape[0] > 0
    q, sx, xr = _act_quant(x)
    oq, osx, oxr = ops.act_quant_had128(x)
    assert torch.equal(xr[tie], oxr[tie])
    assert (xr != oxr).float().mean().item() <= 1e-5
    rq, rs = ops.quantize_rotated(xr)
    assert torch.equal(q, rq) and torch.equal(sx, rs.flatten())
    q2, sx2, _ = _act_quant(x, want_rot=False)
    assert torch.equal(q2, q) and torch.equal(sx2, sx)


@pytest.mark.parametrize("M,K", [(3, 200), (64, 3840), (17, 8), (300, 10240), (1, 10240)])
def test_act_quant_plain_bitexact(cuda, M, K):
    x = seeded_x(M, K, seed=7)
    q, sx, _ = _act_quant(x, had=False, want_rot=False)
    oq, osx = ops.act_quant_plain(x)
    assert torch.equal(q, oq) and torch.equal(sx, osx.flatten())


@pytest.mark.parametrize("K", [3840, 10240, 256])
def test_act_quant_plain_ties_round_half_even(cuda, K):
    """Rows with |max| 127 (x_scale exactly 1) whose values sit on every half-integer tie in
    (-127, 127): the quantiser's integer rounding is round-half-even, as torch.round."""
    ties = torch.arange(-127, 127, dtype=torch.float32) + 0.5
    row = torch.zeros(K)
    row[0] = 127.0
    row[1:1 + ties.numel()] = ties
    row[1 + ties.numel():] = torch.linspace(-126.9, 126.9, K - 1 - ties.numel())
    x = torch.stack([row, -row, row.roll(7)]).to(torch.bfloat16)
    q, sx, _ = _act_quant(x, had=False, want_rot=False)
    oq, osx = ops.act_quant_plain(x)
    assert torch.equal(sx, osx.flatten()) and float(sx[0]) == 1.0
    assert torch.equal(q, oq)


def test_bounded_wait_expires_and_the_context_stays_usable(cuda):
    """A wait that nothing satisfies gives up after its limit and reports ZIB_ERR_TIMEOUT through
    the device error word; the next kernels run normally."""
    assert _lib.device_error_read_clear() == 0
    _lib.call("zib_selftest_bounded_wait", torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert _lib.device_error_read_clear() == _lib.ZIB_ERR_TIMEOUT
    assert _lib.device_error_read_clear() == 0
    x = seeded_x(64, 3840, seed=31)
    q, sx, _ = _act_quant(x, want_rot=False)
    oq, osx, _ = ops.act_quant_had128(x)
    assert torch.equal(q, oq) and torch.equal(sx, osx.flatten())


def _rand_i8(shape, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(-128, 128, shape, generator=g, dtype=torch.int8)


@pytest.fixture(params=[1, 2], ids=["cta1", "cta2"])
def gemm_variant(request):
    """Runs a GEMM test with the 1-CTA (128x256) and the 2-CTA cta_group::2 (256x256) tiling."""
    lib = _lib.load()
    assert lib.zib_gemm_set_variant(request.param) == 0
    yield request.param
    lib.zib_gemm_set_variant(0)


@pytest.mark.parametrize("M,N,K", [(1, 256, 128), (7, 40, 32), (200, 300, 160), (257, 513, 384),
                                   (128, 256, 3840), (300, 1024, 10240), (1024, 11520, 3840),
                                   (2000, 300, 1024)])  # last: A larger than B -> N-blocks-first tile order
def test_gemm_int32_accumulators_bitexact(cuda, gemm_variant, M, N, K):
    q = _rand_i8((M, K), 1)
    w = _rand_i8((N, K), 2)
    acc = torch.empty(M, N + (-N) % 4, dtype=torch.int32, device="cuda")
    qd, wd = q.cuda(), w.cuda()
    _lib.call("zib_gemm_w8a8_acc_i32", qd.data_ptr(), K, wd.data_ptr(), K, acc.data_ptr(), acc.stride(0),
              M, N, K, _lib.stream_of(qd))
    torch.cuda.synchronize()
    assert _lib.device_error_read_clear() == 0
    want = ops.gemm_acc_i32(q, w)
    assert torch.equal(acc[:, :N].cpu(), want)


@pytest.mark.parametrize("M,N,K,bias", [(48, 256, 384, True), (129, 300, 256, False),
                                        (512, 3840, 3840, False), (64, 20480, 3840, True),
                                        (600, 1000, 512, True), (2304, 520, 1024, False)])
def test_gemm_dequant_epilogue_bitexact(cuda, gemm_variant, M, N, K, bias):
    x = seeded_x(M, K, seed=3)
    w = seeded_w(N, K, seed=4)
    wq, sw, _ = ops.weight_prep(w)
    q, sx, _ = ops.act_quant_had128(x)
    b = (torch.randn(N, generator=torch.Generator().manual_seed(5)) * 0.5).to(torch.bfloat16) if bias else None
    ldy = N + (-N) % 8
    y = torch.empty(M, ldy, dtype=torch.bfloat16, device="cuda")
    qd, wd, sxd, swd = q.cuda(), wq.cuda(), sx.flatten().cuda(), sw.cuda()
    bd = b.cuda() if bias else None
    _lib.call("zib_gemm_w8a8", qd.data_ptr(), K, wd.data_ptr(), K, sxd.data_ptr(), swd.data_ptr(),
              _lib.ptr(bd), y.data_ptr(), ldy, M, N, K, _lib.stream_of(qd))
    torch.cuda.synchronize()
    want = ops.dequant_epilogue(ops.gemm_acc_i32(q, wq), sx, sw, b)
    assert torch.equal(y[:, :N].cpu(), want)


@pytest.mark.parametrize("M,N,K", [(1, 256, 128), (2, 46080, 256), (3, 1000, 4096), (5, 300, 160), (8, 4100, 512),
                                   (2, 8, 16)])
def test_gemm_skinny_rows_equal_tensor_core_path(cuda, M, N, K):
    """M <= 8 rows run on the dp4a kernel (automatic variant): bit-identical int32 sums and
    dequant + bias to the tcgen05 path and the oracle."""
    lib = _lib.load()
    q = _rand_i8((M, K), 21)
    w = _rand_i8((N, K), 22)
    g = torch.Generator().manual_seed(23)
    sx = (torch.rand(M, generator=g) * 0.02 + 0.001).to(torch.bfloat16)
    sw = (torch.rand(N, generator=g) * 0.02 + 0.001).to(torch.bfloat16)
    b = (torch.randn(N, generator=g) * 0.5).to(torch.bfloat16)
    qd, wd, sxd, swd, bd = q.cuda(), w.cuda(), sx.cuda(), sw.cuda(), b.cuda()
    st = _lib.stream_of(qd)

    def run(variant, bias):
        assert lib.zib_gemm_set_variant(variant) == 0
        acc = torch.empty(M, N, dtype=torch.int32, device="cuda")
        y = torch.empty(M, N + (-N) % 8, dtype=torch.bfloat16, device="cuda")
        _lib.call("zib_gemm_w8a8_acc_i32", qd.data_ptr(), K, wd.data_ptr(), K, acc.data_ptr(), N, M, N, K, st)
        _lib.call("zib_gemm_w8a8", qd.data_ptr(), K, wd.data_ptr(), K, sxd.data_ptr(), swd.data_ptr(),
                  bd.data_ptr() if bias else None, y.data_ptr(), y.stride(0), M, N, K, st)
        torch.cuda.synchronize()
        assert _lib.device_error_read_clear() == 0
        return acc.cpu(), y[:, :N].cpu()

    try:
        for bias in (False, True):
            a0, y0 = run(0, bias)
            a1, y1 = run(1, bias)
            assert torch.equal(a0, a1) and torch.equal(y0, y1)
            want = ops.gemm_acc_i32(q, w)
            assert torch.equal(a0, want)
            assert torch.equal(y0, ops.dequant_epilogue(want, sx, sw, b if bias else None))
    finally:
        lib.zib_gemm_set_variant(0)


@pytest.mark.parametrize("M,N,K", [(2560, 2048, 6144), (1024, 11520, 10240), (9216, 3840, 10240)])
def test_gemm_split_tail_equals_unsplit(cuda, M, N, K):
    """Short last wave of 2-CTA tiles run as K-split units whose int32 partials the last unit sums:
    identical to the unsplit GEMM (and the oracle), on two calls in a row (the arrival counters
    return to zero), for the int32 and the dequant + bias epilogues."""
    lib = _lib.load()
    q = _rand_i8((M, K), 11)
    w = _rand_i8((N, K), 12)
    sx = (torch.rand(M, generator=torch.Generator().manual_seed(13)) * 0.02 + 0.001).to(torch.bfloat16)
    sw = (torch.rand(N, generator=torch.Generator().manual_seed(14)) * 0.02 + 0.001).to(torch.bfloat16)
    b = (torch.randn(N, generator=torch.Generator().manual_seed(15)) * 0.5).to(torch.bfloat16)
    qd, wd, sxd, swd, bd = q.cuda(), w.cuda(), sx.cuda(), sw.cuda(), b.cuda()
    st = _lib.stream_of(qd)

    def run(split):
        assert lib.zib_gemm_set_split(split) == 0
        acc = torch.empty(M, N, dtype=torch.int32, device="cuda")
        y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        _lib.call("zib_gemm_w8a8_acc_i32", qd.data_ptr(), K, wd.data_ptr(), K, acc.data_ptr(), N, M, N, K, st)
        _lib.call("zib_gemm_w8a8", qd.data_ptr(), K, wd.data_ptr(), K, sxd.data_ptr(), swd.data_ptr(),
                  bd.data_ptr(), y.data_ptr(), N, M, N, K, st)
        torch.cuda.synchronize()
        assert _lib.device_error_read_clear() == 0
        return acc.cpu(), y.cpu()

    try:
        a1, y1 = run(1)
        a2, y2 = run(1)
        a0, y0 = run(0)
        # no registered workspace: the launch runs unsplit
        dev = torch.cuda.current_device()
        assert lib.zib_gemm_set_split_workspace(dev, None, 0, None, 0) == 0
        acc = torch.empty(M, N, dtype=torch.int32, device="cuda")
        assert lib.zib_gemm_set_split(1) == 0
        lib.zib_gemm_w8a8_acc_i32(qd.data_ptr(), K, wd.data_ptr(), K, acc.data_ptr(), N, M, N, K, st)
        torch.cuda.synchronize()
        a3 = acc.cpu()
    finally:
        lib.zib_gemm_set_split(1)
        ws, ctr = _lib._SPLIT_WS[torch.cuda.current_device()]
        lib.zib_gemm_set_split_workspace(torch.cuda.current_device(), ws.data_ptr(), ws.numel() * 4,
                                         ctr.data_ptr(), ctr.numel())
    assert torch.equal(a1, a0) and torch.equal(a2, a0) and torch.equal(a3, a0)
    assert torch.equal(y1, y0) and torch.equal(y2, y0)
    want = ops.gemm_acc_i32(q, w)   # torch._int_mm on the CPU: exact int32 sums
    assert torch.equal(a1, want)
    assert torch.equal(y1, ops.dequant_epilogue(want, sx, sw, b))


@pytest.mark.parametrize("M,F,K", [(48, 128, 384), (129, 384, 256), (300, 1280, 3840), (1024, 10240, 3840),
                                   (1100, 128, 256)])
def test_gemm_swiglu_hadamard_epilogue(cuda, gemm_variant, M, F, K):
    """w1/w3 GEMMs + SwiGLU + w2-input rotation in one launch vs the oracle's composition."""
    x = seeded_x(M, K, seed=13)
    w1q, sw1, _ = ops.weight_prep(seeded_w(F, K, seed=14))
    w3q, sw3, _ = ops.weight_prep(seeded_w(F, K, seed=15))
    q, sx, _ = ops.act_quant_had128(x)
    out = torch.empty(M, F, dtype=torch.bfloat16, device="cuda")
    qd, w1d, w3d, sxd, s1d, s3d = (t.cuda() for t in (q, w1q, w3q, sx.flatten(), sw1, sw3))
    _lib.call("zib_gemm_w8a8_swiglu_had", qd.data_ptr(), K, w1d.data_ptr(), w3d.data_ptr(), K, sxd.data_ptr(),
              s1d.data_ptr(), s3d.data_ptr(), out.data_ptr(), F, M, F, K, _lib.stream_of(qd))
    torch.cuda.synchronize()
    assert _lib.device_error_read_clear() == 0
    g = ops.dequant_epilogue(ops.gemm_acc_i32(q, w1q), sx, sw1, None)
    u = ops.dequant_epilogue(ops.gemm_acc_i32(q, w3q), sx, sw3, None)
    want = ops.rotate_activation_exact(ops.swiglu(g, u))
    got = out.cpu()
    # same fp32 Walsh-Hadamard adds as zib_act_quant: bit-exact but for rare inexact fp32 sums,
    # whose error is a few fp32 ulps of the row's largest partial sum, then one bf16 rounding
    assert (got != want).float().mean().item() <= 1e-5
    rowmax = want.float().abs().amax(dim=1, keepdim=True)
    err = (got.float() - want.float()).abs()
    assert bool((err <= 2 ** -7 * want.float().abs() + 2 ** -16 * rowmax).all()), float(err.max())


def test_gemm_swiglu_matches_composed_kernels(cuda):
    """Fused epilogue == w1/w3 GEMMs, then the SwiGLU + rotation row kernel (bit-exact)."""
    M, F, K = 700, 1024, 3840
    q, sx, _ = ops.act_quant_had128(seeded_x(M, K, seed=21))
    w1q, sw1, _ = ops.weight_prep(seeded_w(F, K, seed=22))
    w3q, sw3, _ = ops.weight_prep(seeded_w(F, K, seed=23))
    qd, sxd = q.cuda(), sx.flatten().cuda()
    w13, s13 = torch.cat([w1q, w3q]).cuda(), torch.cat([sw1, sw3]).cuda()
    st = _lib.stream_of(qd)
    h = torch.empty(M, 2 * F, dtype=torch.bfloat16, device="cuda")
    _lib.call("zib_gemm_w8a8", qd.data_ptr(), K, w13.data_ptr(), K, sxd.data_ptr(), s13.data_ptr(), None,
              h.data_ptr(), 2 * F, M, 2 * F, K, st)
    q_ref = torch.empty(M, F, dtype=torch.int8, device="cuda")
    s_ref = torch.empty(M, dtype=torch.bfloat16, device="cuda")
    _lib.call("zib_swiglu_quant", h.data_ptr(), 2 * F, h.data_ptr() + 2 * F, 2 * F, q_ref.data_ptr(), F,
              s_ref.data_ptr(), M, F, 1, st)
    x_rot = torch.empty(M, F, dtype=torch.bfloat16, device="cuda")
    _lib.call("zib_gemm_w8a8_swiglu_had", qd.data_ptr(), K, w13.data_ptr(), w13.data_ptr() + F * K, K,
              sxd.data_ptr(), s13.data_ptr(), s13.data_ptr() + 2 * F, x_rot.data_ptr(), F, M, F, K, st)
    q_f = torch.empty(M, F, dtype=torch.int8, device="cuda")
    s_f = torch.empty(M, dtype=torch.bfloat16, device="cuda")
    _lib.call("zib_act_quant", x_rot.data_ptr(), F, q_f.data_ptr(), F, s_f.data_ptr(), None, M, F, 0, st)
    torch.cuda.synchronize()
    assert torch.equal(q_f, q_ref) and torch.equal(s_f, s_ref)


@pytest.mark.parametrize("M,F,K", [(48, 128, 384), (129, 384, 256), (1100, 1280, 3840), (2300, 10240, 3840)])
def test_gemm_swiglu_weight_halves_bitexact(cuda, gemm_variant, M, F, K):
    """The one-tensor form ([w1; w3], one 3-D TMA box per CTA and k-block) equals the two-weight
    form bit for bit (same tiles, same epilogue), and both equal the oracle's composed ops."""
    q, sx, _ = ops.act_quant_had128(seeded_x(M, K, seed=41))
    w1q, sw1, _ = ops.weight_prep(seeded_w(F, K, seed=42))
    w3q, sw3, _ = ops.weight_prep(seeded_w(F, K, seed=43))
    qd, w1d, w3d, sxd, s1d, s3d = (t.cuda() for t in (q, w1q, w3q, sx.flatten(), sw1, sw3))
    st = _lib.stream_of(qd)
    w13 = torch.cat([w1d, w3d], 0)
    ref = torch.empty(M, F, dtype=torch.bfloat16, device="cuda")
    _lib.call("zib_gemm_w8a8_swiglu_had", qd.data_ptr(), K, w1d.data_ptr(), w3d.data_ptr(), K, sxd.data_ptr(),
              s1d.data_ptr(), s3d.data_ptr(), ref.data_ptr(), F, M, F, K, st)
    got = torch.empty(M, F, dtype=torch.bfloat16, device="cuda")
    for _ in range(2):
        got.fill_(0)
        _lib.call("zib_gemm_w8a8_swiglu_had_w13", qd.data_ptr(), K, w13.data_ptr(), K, sxd.data_ptr(),
                  s1d.data_ptr(), s3d.data_ptr(), got.data_ptr(), F, M, F, K, st)
        torch.cuda.synchronize()
        assert _lib.device_error_read_clear() == 0
        assert torch.equal(got, ref)
    g = ops.dequant_epilogue(ops.gemm_acc_i32(q, w1q), sx, sw1, None)
    u = ops.dequant_epilogue(ops.gemm_acc_i32(q, w3q), sx, sw3, None)
    want = ops.rotate_activation_exact(ops.swiglu(g, u))
    # the epilogue's Hadamard sums are fp32 (the exact-sum oracle rounds once): rare 1-ulp differences
    assert (ref.cpu() != want).float().mean().item() <= 1e-5


def test_gemm_swiglu_rejects_ragged_features(cuda):
    q = torch.zeros(8, 128, dtype=torch.int8, device="cuda")
    w = torch.zeros(200, 128, dtype=torch.int8, device="cuda")
    s = torch.ones(256, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(8, 200, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="group_size"):
        _lib.call("zib_gemm_w8a8_swiglu_had", q.data_ptr(), 128, w.data_ptr(), w.data_ptr(), 128, s.data_ptr(),
                  s.data_ptr(), s.data_ptr(), out.data_ptr(), 200, 8, 200, 128, _lib.stream_of(q))


@pytest.mark.parametrize("B,S,H,fb", [(2, 48, 2, 1), (1, 200, 4, 1), (2, 130, 30, 2)])
def test_gemm_qk_norm_rope_epilogue_bitexact(cuda, gemm_variant, B, S, H, fb):
    """QKV GEMM + per-head RMSNorm + RoPE on Q and K in one launch vs GEMM then fused_qknorm_rope."""
    from zimage_b200.kernels.fused_qknorm_rope import rope_tables

    M, K, N = B * S, 384 if H < 30 else 3840, 3 * H * 128
    x = seeded_x(M, K, seed=17)
    wq, sw, _ = ops.weight_prep(seeded_w(N, K, seed=18))
    q, sx, _ = ops.act_quant_had128(x)
    qw, kw = _norm_w(128, 19), _norm_w(128, 20)
    pos = ops.zimage_positions(8, 8, S)[:S]
    fc = ops.rope_freqs_complex(pos).unsqueeze(0).expand(fb, -1, -1).contiguous()
    if fb == 2:
        fc[1] = fc[1].conj()  # a different table per batch entry
    cos, sin, cs_b = rope_tables(fc.cuda(), B)
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    qd, wd, sxd, swd = q.cuda(), wq.cuda(), sx.flatten().cuda(), sw.cuda()
    qwd, kwd = qw.float().cuda(), kw.float().cuda()
    _lib.call("zib_gemm_w8a8_qk_norm_rope", qd.data_ptr(), K, wd.data_ptr(), K, sxd.data_ptr(), swd.data_ptr(),
              y.data_ptr(), N, M, N, K, qwd.data_ptr(), kwd.data_ptr(), 1e-5, 1e-6, cos.data_ptr(),
              sin.data_ptr(), cs_b, S, H, _lib.stream_of(qd))
    torch.cuda.synchronize()
    assert _lib.device_error_read_clear() == 0
    plain = ops.dequant_epilogue(ops.gemm_acc_i32(q, wq), sx, sw, None).reshape(B, S, 3, H, 128)
    got = y.cpu().reshape(B, S, 3, H, 128)
    assert torch.equal(got[:, :, 0], ops.fused_qknorm_rope(plain[:, :, 0], qw, fc, 1e-5))
    assert torch.equal(got[:, :, 1], ops.fused_qknorm_rope(plain[:, :, 1], kw, fc, 1e-6))
    assert torch.equal(got[:, :, 2], plain[:, :, 2])


def test_gemm_qk_norm_rope_rejects_odd_heads(cuda):
    q = torch.zeros(8, 128, dtype=torch.int8, device="cuda")
    w = torch.zeros(3 * 3 * 128, 128, dtype=torch.int8, device="cuda")
    s = torch.ones(3 * 3 * 128, dtype=torch.bfloat16, device="cuda")
    f = torch.ones(8 * 64, dtype=torch.float32, device="cuda")
    y = torch.empty(8, 3 * 3 * 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="even head count"):
        _lib.call("zib_gemm_w8a8_qk_norm_rope", q.data_ptr(), 128, w.data_ptr(), 128, s.data_ptr(), s.data_ptr(),
                  y.data_ptr(), 3 * 3 * 128, 8, 3 * 3 * 128, 128, f.data_ptr(), f.data_ptr(), 1e-5, 1e-5,
                  f.data_ptr(), f.data_ptr(), 0, 8, 3, _lib.stream_of(q))


@pytest.mark.parametrize("N,K,had", [(256, 384, True), (64, 176, False), (1000, 3840, True), (40, 10240, True)])
def test_weight_prep_bitexact(cuda, N, K, had):
    w = seeded_w(N, K, seed=N)
    wd = w.cuda()
    wq = torch.empty(N, K, dtype=torch.int8, device="cuda")
    sw = torch.empty(N, dtype=torch.bfloat16, device="cuda")
    sw32 = torch.empty(N, dtype=torch.float32, device="cuda")
    rot = torch.empty(N, K, dtype=torch.float32, device="cuda")
    _lib.call("zib_weight_prep", wd.data_ptr(), K, wq.data_ptr(), K, sw.data_ptr(), sw32.data_ptr(),
              rot.data_ptr(), K, N, K, 1 if had else 0, _lib.stream_of(wd))
    torch.cuda.synchronize()
    owq, osw, osw32 = ops.weight_prep(w, hadamard=had)
    assert torch.equal(wq.cpu(), owq)
    assert torch.equal(sw.cpu(), osw)
    assert torch.equal(sw32.cpu(), osw32)
    want_rot = ops.rotate_weight_exact(w) if had else w.float()
    assert torch.equal(rot.cpu(), want_rot)


# ---------------------------------------------------------------------------
# row kernels
# ---------------------------------------------------------------------------

def _norm_w(n, seed=11):
    return (1.0 + 0.1 * torch.randn(n, generator=torch.Generator().manual_seed(seed))).to(torch.bfloat16)


@pytest.mark.parametrize("shape", [(2, 7, 3840), (1, 1, 128), (3, 5, 1000), (4, 130)])
def test_rms_norm_bitexact(cuda, shape):
    from zimage_b200 import triton_rms_norm

    x = seeded_x(int(torch.tensor(shape[:-1]).prod()), shape[-1], seed=9).reshape(shape)
    w = _norm_w(shape[-1])
    y = triton_rms_norm(x.cuda(), w.cuda(), eps=1e-5).cpu()
    assert torch.equal(y, ops.rms_norm(x, w, 1e-5))


def test_rmsnorm_mod_and_quant_bitexact(cuda):
    B, S, D = 2, 33, 3840
    x = seeded_x(B * S, D, seed=12).reshape(B, S, D)
    w = _norm_w(D)
    raw = (torch.randn(B, 4 * D, generator=torch.Generator().manual_seed(13)) * 0.1).to(torch.bfloat16)
    scale = raw[:, :D]
    want = ops.modulate(ops.rms_norm(x, w, 1e-5), scale)
    xd, wd, rawd = x.cuda().contiguous(), w.float().cuda(), raw.cuda()
    y = torch.empty(B * S, D, dtype=torch.bfloat16, device="cuda")
    st = _lib.stream_of(xd)
    _lib.call("zib_rmsnorm_mod", xd.data_ptr(), D, wd.data_ptr(), rawd.data_ptr(), None, 4 * D, S,
              y.data_ptr(), D, B * S, D, 1e-5, st)
    q = torch.empty(B * S, D, dtype=torch.int8, device="cuda")
    sx = torch.empty(B * S, dtype=torch.bfloat16, device="cuda")
    _lib.call("zib_rmsnorm_mod_quant", xd.data_ptr(), D, wd.data_ptr(), rawd.data_ptr(), None, 4 * D, S,
              q.data_ptr(), D, sx.data_ptr(), B * S, D, 1e-5, 1, st)
    torch.cuda.synchronize()
    assert torch.equal(y.cpu().reshape(B, S, D), want)
    oq, osx, _ = ops.act_quant_had128(want.reshape(B * S, D))
    assert torch.equal(sx.cpu(), osx.flatten())
    assert torch.equal(q.cpu(), oq)


@pytest.mark.parametrize("had,with_shift", [(False, True), (True, True)])
def test_rmsnorm_mod_quant_shift_and_plain_bitexact(cuda, had, with_shift):
    """The 3840-wide norm + modulation + quantisation (quad-layout kernel) over 500 rows of two
    batches, with the shift, with and without the rotation."""
    B, S, D = 2, 250, 3840
    x = seeded_x(B * S, D, seed=14).reshape(B, S, D)
    w = _norm_w(D, 15)
    gen = torch.Generator().manual_seed(16)
    scale = (torch.randn(B, D, generator=gen) * 0.1).to(torch.bfloat16)
    shift = (torch.randn(B, D, generator=gen) * 0.1).to(torch.bfloat16) if with_shift else None
    want = ops.modulate(ops.rms_norm(x, w, 1e-5), scale, shift).reshape(B * S, D)
    oq, osx = ops.act_quant_had128(want)[:2] if had else ops.act_quant_plain(want)
    xd, wd, sd = x.cuda().contiguous(), w.float().cuda(), scale.cuda()
    hd = None if shift is None else shift.cuda()
    q = torch.empty(B * S, D, dtype=torch.int8, device="cuda")
    sx = torch.empty(B * S, dtype=torch.bfloat16, device="cuda")
    _lib.call("zib_rmsnorm_mod_quant", xd.data_ptr(), D, wd.data_ptr(), sd.data_ptr(),
              None if hd is None else hd.data_ptr(), D, S, q.data_ptr(), D, sx.data_ptr(), B * S, D, 1e-5,
              1 if had else 0, _lib.stream_of(xd))
    torch.cuda.synchronize()
    assert torch.equal(sx.cpu(), osx.flatten())
    assert torch.equal(q.cpu(), oq)


def test_norm_gate_residual_and_fused_quant_bitexact(cuda):
    from zimage_b200 import triton_fused_norm_gate_residual

    B, S, D = 2, 17, 3840
    x = seeded_x(B * S, D, seed=21).reshape(B, S, D)
    r = seeded_x(B * S, D, seed=22).reshape(B, S, D)
    g = torch.tanh(torch.randn(B, 1, D, generator=torch.Generator().manual_seed(23))).to(torch.bfloat16)
    w, w2 = _norm_w(D, 1), _norm_w(D, 2)
    want = ops.norm_gate_residual(x, r, g, w, 1e-5)
    y = triton_fused_norm_gate_residual(x.cuda(), r.cuda(), g.cuda(), w.cuda(), 1e-5).cpu()
    assert torch.equal(y, want)
    # fused with the next norm + modulation + quantisation
    s = (torch.randn(B, D, generator=torch.Generator().manual_seed(24)) * 0.1).to(torch.bfloat16)
    xd, rd, gd, sd = x.cuda().contiguous(), r.cuda().contiguous(), g.reshape(B, D).cuda().contiguous(), s.cuda()
    wd, w2d = w.float().cuda(), w2.float().cuda()
    y2 = torch.empty(B * S, D, dtype=torch.bfloat16, device="cuda")
    q = torch.empty(B * S, D, dtype=torch.int8, device="cuda")
    sx = torch.empty(B * S, dtype=torch.bfloat16, device="cuda")
    _lib.call("zib_norm_gate_residual_mod_quant", xd.data_ptr(), D, rd.data_ptr(), D, gd.data_ptr(), D, S,
              wd.data_ptr(), y2.data_ptr(), D, w2d.data_ptr(), sd.data_ptr(), None, D,
              q.data_ptr(), D, sx.data_ptr(), B * S, D, 1e-5, 1e-6, 1, _lib.stream_of(xd))
    torch.cuda.synchronize()
    assert torch.equal(y2.cpu().reshape(B, S, D), want)
    nxt = ops.modulate(ops.rms_norm(want, w2, 1e-6), s)
    oq, osx, _ = ops.act_quant_had128(nxt.reshape(B * S, D))
    assert torch.equal(sx.cpu(), osx.flatten())
    assert torch.equal(q.cpu(), oq)


@pytest.mark.parametrize("rows,had,with_shift", [(1, True, False), (600, True, True), (257, False, False)])
def test_norm_gate_residual_mod_quant_rows_bitexact(cuda, rows, had, with_shift):
    """The fused norm kernel at the step width (3840, the register-resident kernel) over many
    rows of two batches, with and without the rotation and the shift."""
    D = 3840
    B = 2 if rows > 1 else 1
    per = (rows + B - 1) // B
    x = seeded_x(rows, D, seed=41 + rows)
    r = seeded_x(rows, D, seed=42 + rows)
    x[0] *= 300.0  # a large row next to ordinary ones
    gen = torch.Generator().manual_seed(43)
    g = torch.tanh(torch.randn(B, D, generator=gen)).to(torch.bfloat16)
    s = (torch.randn(B, D, generator=gen) * 0.1).to(torch.bfloat16)
    h = (torch.randn(B, D, generator=gen) * 0.1).to(torch.bfloat16) if with_shift else None
    w, w2 = _norm_w(D, 5), _norm_w(D, 6)
    bidx = torch.arange(rows) // per
    # each row as its own [1, 1, D] batch item of the oracle, with its batch's vectors
    want = ops.norm_gate_residual(x.reshape(rows, 1, D), r.reshape(rows, 1, D), g[bidx], w, 1e-5)
    nxt = ops.modulate(ops.rms_norm(want, w2, 1e-6), s[bidx], None if h is None else h[bidx])
    want, nxt = want.reshape(rows, D), nxt.reshape(rows, D)
    oq, osx = ops.act_quant_had128(nxt)[:2] if had else ops.act_quant_plain(nxt)
    xd, rd, gd, sd = x.cuda(), r.cuda(), g.cuda(), s.cuda()
    hd = None if h is None else h.cuda()
    wd, w2d = w.float().cuda(), w2.float().cuda()
    y = torch.empty(rows, D, dtype=torch.bfloat16, device="cuda")
    q = torch.empty(rows, D, dtype=torch.int8, device="cuda")
    sx = torch.empty(rows, dtype=torch.bfloat16, device="cuda")
    _lib.call("zib_norm_gate_residual_mod_quant", xd.data_ptr(), D, rd.data_ptr(), D, gd.data_ptr(), D, per,
              wd.data_ptr(), y.data_ptr(), D, w2d.data_ptr(), sd.data_ptr(),
              None if hd is None else hd.data_ptr(), D, q.data_ptr(), D, sx.data_ptr(), rows, D, 1e-5, 1e-6,
              1 if had else 0, _lib.stream_of(xd))
    torch.cuda.synchronize()
    assert torch.equal(y.cpu(), want)
    assert torch.equal(sx.cpu(), osx.flatten())
    assert torch.equal(q.cpu(), oq)


@pytest.mark.parametrize("M,N,K,budget", [(1536, 2304, 512, 1 << 18), (1792, 2304, 512, 3 << 17),
                                          (2048, 1024, 768, 1 << 18), (700, 4096, 384, 1 << 17),
                                          (384, 768, 256, 0)])
def test_gemm_grouped_tile_order_bitexact(cuda, gemm_variant, M, N, K, budget):
    """Tile orders that sweep the re-read operand in groups (a small L2 budget forces several
    groups of balanced and unbalanced sizes, both operand orders): the same int32 accumulators
    and outputs as the oracle."""
    lib = _lib.load()
    q, w = _rand_i8((M, K), 71 + M), _rand_i8((N, K), 72 + N)
    try:
        assert lib.zib_gemm_set_group_budget(budget) == 0
        acc = torch.empty(M, N, dtype=torch.int32, device="cuda")
        qd, wd = q.cuda(), w.cuda()
        _lib.call("zib_gemm_w8a8_acc_i32", qd.data_ptr(), K, wd.data_ptr(), K, acc.data_ptr(), N, M, N, K,
                  _lib.stream_of(qd))
        torch.cuda.synchronize()
    finally:
        assert lib.zib_gemm_set_group_budget(0) == 0
    assert torch.equal(acc.cpu(), ops.gemm_acc_i32(q, w))


@pytest.mark.parametrize("had,with_shift", [(True, False), (False, True)])
def test_norm_gate_residual_mod_quant_bf16_weights_equal_fp32(cuda, had, with_shift):
    """The bf16-weight entry gives the fp32 entry's outputs for the same (bf16-valued) weights."""
    rows, D, S = 700, 3840, 350
    x, r = seeded_x(rows, D, seed=81).cuda(), seeded_x(rows, D, seed=82).cuda()
    gen = torch.Generator().manual_seed(83)
    g = torch.tanh(torch.randn(2, D, generator=gen)).to(torch.bfloat16).cuda()
    sc = (torch.randn(2, D, generator=gen) * 0.1).to(torch.bfloat16).cuda()
    sh = (torch.randn(2, D, generator=gen) * 0.1).to(torch.bfloat16).cuda() if with_shift else None
    w, w2 = _norm_w(D, 84).cuda(), _norm_w(D, 85).cuda()
    outs = []
    for entry, wa, wb in (("zib_norm_gate_residual_mod_quant", w.float(), w2.float()),
                          ("zib_norm_gate_residual_mod_quant_w16", w, w2)):
        y = torch.empty(rows, D, dtype=torch.bfloat16, device="cuda")
        q = torch.empty(rows, D, dtype=torch.int8, device="cuda")
        sx = torch.empty(rows, dtype=torch.bfloat16, device="cuda")
        _lib.call(entry, x.data_ptr(), D, r.data_ptr(), D, g.data_ptr(), D, S, wa.data_ptr(), y.data_ptr(), D,
                  wb.data_ptr(), sc.data_ptr(), None if sh is None else sh.data_ptr(), D, q.data_ptr(), D,
                  sx.data_ptr(), rows, D, 1e-5, 1e-6, 1 if had else 0, _lib.stream_of(x))
        torch.cuda.synchronize()
        outs.append((y.cpu(), q.cpu(), sx.cpu()))
    for a, b in zip(*outs):
        assert torch.equal(a, b)
    with pytest.raises(ValueError):  # other row widths are refused
        _lib.call("zib_norm_gate_residual_mod_quant_w16", x.data_ptr(), 1024, r.data_ptr(), 1024, g.data_ptr(),
                  1024, S, w.data_ptr(), x.data_ptr(), 1024, w2.data_ptr(), sc.data_ptr(), None, 1024,
                  x.data_ptr(), 1024, x.data_ptr(), rows, 1024, 1e-5, 1e-6, 1, _lib.stream_of(x))


def test_swiglu_silu_on_every_bf16_gate(cuda):
    """bf16(bf16(silu(g)) * 1) for every finite bf16 gate g (all 65,280 of them) equals the
    oracle's fp32 SiLU rounded to bf16: the kernels' SiLU is exact on its whole input domain."""
    import numpy as np

    g = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    g = g[torch.isfinite(g.float())].reshape(255, 256)  # 256-wide rows: the warp-per-row kernel's form
    up = torch.ones_like(g)
    out = torch.empty_like(g, device="cuda")
    gd, ud = g.cuda(), up.cuda()
    _lib.call("zib_swiglu", gd.data_ptr(), 256, ud.data_ptr(), 256, out.data_ptr(), 256, 255, 256,
              _lib.stream_of(gd))
    torch.cuda.synchronize()
    gf = g.float().numpy()
    with np.errstate(over="ignore"):
        want = torch.from_numpy((gf * ops.sigmoid_f32(gf)).astype(np.float32)).to(torch.bfloat16)
    bad = (out.cpu() != want).nonzero()
    assert bad.numel() == 0, [(float(g[i, j]), float(out[i, j]), float(want[i, j])) for i, j in bad[:8]]


def test_swiglu_and_fused_quant(cuda):
    from zimage_b200 import triton_swiglu_forward

    M, F = 40, 10240
    gate = seeded_x(M, F, seed=31, outlier_frac=0.0)
    up = seeded_x(M, F, seed=32, outlier_frac=0.0)
    out = triton_swiglu_forward(gate.cuda(), up.cuda()).cpu()
    want = ops.swiglu(gate, up)
    # sigmoid is an fp32 library function on both sides: rare 1-ulp bf16 differences
    assert (out != want).float().mean().item() < 1e-3
    assert (out.float() - want.float()).abs().max().item() <= 2 ** -6 * want.float().abs().max().item()
    h = torch.cat([gate, up], dim=1).cuda()
    q = torch.empty(M, F, dtype=torch.int8, device="cuda")
    sx = torch.empty(M, dtype=torch.bfloat16, device="cuda")
    _lib.call("zib_swiglu_quant", h.data_ptr(), 2 * F, h.data_ptr() + 2 * F, 2 * F, q.data_ptr(), F,
              sx.data_ptr(), M, F, 1, _lib.stream_of(h))
    torch.cuda.synchronize()
    oq, osx, _ = ops.act_quant_had128(out)  # quantisation of the kernel's own SwiGLU output
    assert torch.equal(sx.cpu(), osx.flatten())
    assert torch.equal(q.cpu(), oq)


@pytest.mark.parametrize("B,S,H,fb", [(2, 48, 30, 1), (1, 5, 3, 1), (2, 9, 4, 2)])
def test_qknorm_rope_bitexact(cuda, B, S, H, fb):
    from zimage_b200 import triton_fused_qknorm_rope, triton_rope_3d

    x = seeded_x(B * S * H, 128, seed=41).reshape(B, S, H, 128)
    w = _norm_w(128, 42)
    pos = ops.zimage_positions(4, 4, S)[:S]
    fc = ops.rope_freqs_complex(pos).unsqueeze(0).expand(fb, -1, -1).contiguous()
    want = ops.fused_qknorm_rope(x, w, fc, 1e-6)
    got = triton_fused_qknorm_rope(x.cuda(), w.cuda(), fc.cuda(), eps=1e-6).cpu()
    assert torch.equal(got, want)
    want_r = ops.rope_3d(x, fc)
    got_r = triton_rope_3d(x.cuda(), fc.cuda()).cpu()
    assert torch.equal(got_r, want_r)


def test_qknorm_rope_strided_in_place(cuda):
    """In place on the Q slice of a fused QKV buffer (the block's use)."""
    from zimage_b200.kernels.fused_qknorm_rope import qknorm_rope_into, rope_tables

    B, S, H = 2, 16, 30
    qkv = seeded_x(B * S, 3 * H * 128, seed=51).reshape(B, S, 3, H, 128)
    w = _norm_w(128, 52)
    fc = ops.rope_freqs_complex(ops.zimage_positions(4, 4, 0)).unsqueeze(0)
    want = ops.fused_qknorm_rope(qkv[:, :, 1], w, fc, 1e-5)
    d = qkv.cuda()
    xk = d[:, :, 1]
    cos, sin, cs_b = rope_tables(fc.cuda(), B)
    qknorm_rope_into(xk, xk, w.float().cuda(), cos, sin, cs_b, 1e-5)
    torch.cuda.synchronize()
    got = d.cpu()
    assert torch.equal(got[:, :, 1], want)
    assert torch.equal(got[:, :, 0], qkv[:, :, 0]) and torch.equal(got[:, :, 2], qkv[:, :, 2])


def test_adaln_kernels(cuda):
    from zimage_b200 import triton_adaln_modulation

    B, D = 2, 3840
    raw = (torch.randn(B, 4 * D, generator=torch.Generator().manual_seed(61)) * 0.5).to(torch.bfloat16)
    got = triton_adaln_modulation(raw.cuda(), D)
    want = ops.adaln_modulation(raw, D)
    for a, b in zip(got, want):
        a = a.cpu()
        assert (a != b).float().mean().item() < 1e-3
        assert (a.float() - b.float()).abs().max().item() <= 2 ** -7
    gates = torch.empty(B, 2, D, dtype=torch.bfloat16, device="cuda")
    rd = raw.cuda()
    _lib.call("zib_adaln_gates", rd.data_ptr(), 4 * D, gates.data_ptr(), B, D, _lib.stream_of(rd))
    torch.cuda.synchronize()
    assert torch.equal(gates[:, 0].cpu(), got[1].cpu()) and torch.equal(gates[:, 1].cpu(), got[3].cpu())
