"""zib_gemm_w8a8_static_scratch against zib_gemm_w8a8, through the C ABI (needs a B200).

The static-scratch GEMM is for callers that must not allocate device memory (a framework
that budgets the GPU's memory through its own pool, a stream capture in progress, a
latency-bound loop where cudaMalloc would synchronise): its split-K partials live in a fixed
16 MB static device area instead of a workspace that the caller allocates and registers.

Kept in its own file so that it is collected last: it must pass alone and after the rest
of the suite, with whatever the earlier tests left in the static scratch.
"""

import pytest
import torch

from zimage_b200 import _lib

pytestmark = pytest.mark.gpu

STATIC_UNITS = 64  # units of 2 x 128 x 256 int32 partials in the static scratch


def _operands(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randint(-128, 128, (M, K), generator=g, dtype=torch.int8).cuda()
    w = torch.randint(-128, 128, (N, K), generator=g, dtype=torch.int8).cuda()
    sx = (torch.rand(M, generator=g) * 0.02 + 0.001).to(torch.bfloat16).cuda()
    sw = (torch.rand(N, generator=g) * 0.02 + 0.001).to(torch.bfloat16).cuda()
    b = (torch.randn(N, generator=g) * 0.5).to(torch.bfloat16).cuda()
    return q, w, sx, sw, b


def _tail_tiles(M, N):
    """Tiles in the short last wave of a 2-CTA launch (0 when there is none)."""
    pairs = torch.cuda.get_device_properties(0).multi_processor_count // 2
    tiles = ((M + 255) // 256) * ((N + 255) // 256)
    return 0 if tiles <= pairs else tiles % pairs


def _gemm(name, q, w, sx, sw, b, M, N, K, *extra):
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    _lib.call(name, q.data_ptr(), K, w.data_ptr(), K, sx.data_ptr(), sw.data_ptr(), b.data_ptr(), y.data_ptr(),
              N, M, N, K, *extra, _lib.stream_of(q))
    return y


@pytest.mark.parametrize("M,N,K,splits", [(9216, 3840, 10240, 2), (2560, 2048, 6144, 3), (1024, 11520, 3840, 2),
                                          (2560, 2048, 6144, 1)])
def test_static_scratch_gemm_equals_allocating_gemm(cuda, M, N, K, splits):
    if _tail_tiles(M, N) * splits > STATIC_UNITS:
        pytest.skip(f"the last wave of {M}x{N} on this GPU's SM count does not fit the static scratch")
    q, w, sx, sw, b = _operands(M, N, K, seed=M + N + K)
    want = _gemm("zib_gemm_w8a8", q, w, sx, sw, b, M, N, K)
    first = _gemm("zib_gemm_w8a8_static_scratch", q, w, sx, sw, b, M, N, K, splits)
    second = _gemm("zib_gemm_w8a8_static_scratch", q, w, sx, sw, b, M, N, K, splits)
    torch.cuda.synchronize()
    assert _lib.device_error_read_clear() == 0
    assert torch.equal(first, want)
    assert torch.equal(second, want)


def test_static_scratch_calls_leave_free_device_memory_unchanged(cuda):
    """After the first call on the device (which looks up the scratch address), calls take
    no device memory: the free memory the driver reports is the same before and after."""
    M, N, K = 9216, 3840, 10240
    q, w, sx, sw, b = _operands(M, N, K, seed=11)
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    args = (q.data_ptr(), K, w.data_ptr(), K, sx.data_ptr(), sw.data_ptr(), b.data_ptr(), y.data_ptr(), N, M, N, K,
            2, _lib.stream_of(q))
    _lib.call("zib_gemm_w8a8_static_scratch", *args)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        _lib.call("zib_gemm_w8a8_static_scratch", *args)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert torch.equal(y, _gemm("zib_gemm_w8a8", q, w, sx, sw, b, M, N, K))


def test_static_scratch_reaches_the_split_planner(cuda):
    """A short last wave with more splits than 128-wide K-blocks is refused by the split
    planner (so the split path is the one these shapes take), before any launch."""
    M, N, K = 2560, 2048, 256
    if _tail_tiles(M, N) == 0:
        pytest.skip("no short last wave on this GPU's SM count")
    q, w, sx, sw, b = _operands(M, N, K, seed=13)
    with pytest.raises(ValueError, match="exceed the 2 K-blocks"):
        _gemm("zib_gemm_w8a8_static_scratch", q, w, sx, sw, b, M, N, K, 3)
    got = _gemm("zib_gemm_w8a8_static_scratch", q, w, sx, sw, b, M, N, K, 2)
    torch.cuda.synchronize()
    assert torch.equal(got, _gemm("zib_gemm_w8a8", q, w, sx, sw, b, M, N, K))


def test_static_scratch_refuses_a_tail_larger_than_the_scratch(cuda):
    M, N, K, splits = 9216, 3840, 10240, 3
    tail = _tail_tiles(M, N)
    q, w, sx, sw, b = _operands(M, N, K, seed=5)
    if tail * splits <= STATIC_UNITS:
        pytest.skip(f"{tail} tail tiles x {splits} splits fit this GPU's SM count")
    with pytest.raises(RuntimeError, match="split-K scratch"):
        _gemm("zib_gemm_w8a8_static_scratch", q, w, sx, sw, b, M, N, K, splits)
    # refused before any launch: the next call still matches the allocating GEMM
    want = _gemm("zib_gemm_w8a8", q, w, sx, sw, b, M, N, K)
    got = _gemm("zib_gemm_w8a8_static_scratch", q, w, sx, sw, b, M, N, K, 2)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


@pytest.mark.parametrize("splits", [0, 5])
def test_static_scratch_rejects_bad_split_counts(cuda, splits):
    q, w, sx, sw, b = _operands(256, 256, 256, seed=7)
    with pytest.raises(ValueError, match="splits must be 1 to 4"):
        _gemm("zib_gemm_w8a8_static_scratch", q, w, sx, sw, b, 256, 256, 256, splits)
