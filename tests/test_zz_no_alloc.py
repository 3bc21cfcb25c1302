"""The allocation-free quantize entry point (fp8b200_quantize_fp8_noalloc).

It exists for callers that cannot allocate device memory where they
quantise (a host runtime that owns all device memory and passes the library
only the tensors to read and write). Its scratch is a fixed array inside the
library, so this test checks, through the C ABI, that it gives exactly what
the allocating entry point gives, on two calls in a row (the second call must
not see the first call's leftovers), and that it refuses inputs larger than
its fixed scratch can cover.

This file is collected last so that a run stopping at the first failure has
already run every other test.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

CODE = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


def _allocating(L, x, fmt):
    out = torch.empty(x.numel(), dtype=torch.uint8, device="cuda")
    scales = torch.empty(2, dtype=torch.float32, device="cuda")
    scratch = torch.empty(1, dtype=torch.int32, device="cuda")
    L.check(L.lib().fp8b200_quantize_fp8(x.data_ptr(), CODE[x.dtype], out.data_ptr(), fmt, x.numel(),
                                         scales.data_ptr(), scratch.data_ptr(),
                                         torch.cuda.current_stream().cuda_stream), "quantize")
    return out, scales


def _noalloc(L, x, fmt):
    out = torch.empty(x.numel(), dtype=torch.uint8, device="cuda")
    scales = torch.empty(2, dtype=torch.float32, device="cuda")
    L.check(L.lib().fp8b200_quantize_fp8_noalloc(x.data_ptr(), CODE[x.dtype], out.data_ptr(), fmt, x.numel(),
                                                 scales.data_ptr(), torch.cuda.current_stream().cuda_stream),
            "quantize_noalloc")
    return out, scales


@pytest.fixture(scope="module")
def L(device):
    import ctypes
    from fp4_fp8_for_torch_mps import _lib
    lib = _lib.lib()
    lib.fp8b200_quantize_fp8_noalloc.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                                 ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
    lib.fp8b200_quantize_fp8_noalloc.restype = ctypes.c_int
    return _lib


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("fmt", [3, 4])
def test_matches_allocating_entry_point_on_two_calls(L, dtype, fmt):
    g = torch.Generator().manual_seed(17)
    # call 1: large tensor with a large amax spread over many scratch slices;
    # call 2: smaller tensor with a smaller amax, so stale partials from call 1
    # would change its scale if they leaked into it
    big = (torch.randn(3 * 65536 + 1234, generator=g) * 300).to(dtype).cuda()
    small = (torch.randn(70000, generator=g) * 2).to(dtype).cuda()
    for x in (big, small):
        ref_codes, ref_scales = _allocating(L, x, fmt)
        got_codes, got_scales = _noalloc(L, x, fmt)
        torch.cuda.synchronize()
        assert torch.equal(got_scales.cpu(), ref_scales.cpu())
        assert torch.equal(got_codes.cpu(), ref_codes.cpu())


def test_special_values_and_empty(L):
    x = torch.tensor([0.0, -0.0, 1.0, -3.5, float("nan"), 2.0], device="cuda")
    for t in (x, torch.zeros(10, device="cuda"), torch.empty(0, device="cuda")):
        rc, rs = _allocating(L, t, 3)
        gc, gs = _noalloc(L, t, 3)
        torch.cuda.synchronize()
        assert np.array_equal(gs.cpu().numpy().view(np.uint32), rs.cpu().numpy().view(np.uint32))
        assert torch.equal(gc.cpu(), rc.cpu())


def test_rejects_inputs_beyond_its_scratch(L):
    lib = L.lib()
    limit = 4096 * 65536
    x = torch.zeros(16, device="cuda")
    out = torch.empty(16, dtype=torch.uint8, device="cuda")
    scales = torch.empty(2, device="cuda")
    # the size check runs before any memory is touched
    rc = lib.fp8b200_quantize_fp8_noalloc(x.data_ptr(), 0, out.data_ptr(), 3, limit + 1, scales.data_ptr(),
                                          torch.cuda.current_stream().cuda_stream)
    assert rc == -1
    assert b"exceed the limit" in lib.fp8b200_last_error()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_unaligned_view(L, dtype):
    """A view one element into its storage (not 16-byte aligned) takes the
    element-by-element amax and encode paths; results still match."""
    g = torch.Generator().manual_seed(3)
    base = (torch.randn(5 * 65536 + 77, generator=g) * 50).to(dtype).cuda()
    x = base[1:]
    assert x.data_ptr() % 16 != 0
    rc, rs = _allocating(L, x, 3)
    gc, gs = _noalloc(L, x, 3)
    torch.cuda.synchronize()
    assert torch.equal(gs.cpu(), rs.cpu()) and torch.equal(gc.cpu(), rc.cpu())


def test_graph_capture_and_replay(L):
    """After a first (warm) call on the device, the entry point can be captured
    in a CUDA graph; each replay equals an eager call on the current input."""
    g = torch.Generator().manual_seed(9)
    x = (torch.randn(200_000, generator=g) * 10).cuda()
    _noalloc(L, x, 3)  # first call on the device before any capture
    torch.cuda.synchronize()
    out = torch.empty(x.numel(), dtype=torch.uint8, device="cuda")
    scales = torch.empty(2, dtype=torch.float32, device="cuda")
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            L.check(L.lib().fp8b200_quantize_fp8_noalloc(x.data_ptr(), 0, out.data_ptr(), 3, x.numel(),
                                                         scales.data_ptr(), side.cuda_stream), "capture")
    for scale in (1.0, 0.01):
        x.mul_(scale)
        graph.replay()
        torch.cuda.synchronize()
        rc, rs = _allocating(L, x, 3)
        torch.cuda.synchronize()
        assert torch.equal(scales.cpu(), rs.cpu()) and torch.equal(out.cpu(), rc.cpu())


def test_at_the_size_limit(L):
    """Exactly FP8B200_NOALLOC_MAX_ELEMENTS bf16 elements (512 MiB, all 4096
    scratch slices), the largest amax in the last slice."""
    limit = 4096 * 65536
    x = torch.empty(limit, dtype=torch.bfloat16, device="cuda")
    x.normal_(generator=torch.Generator(device="cuda").manual_seed(1))
    x[-5] = 1000.0
    rc, rs = _allocating(L, x, 3)
    gc, gs = _noalloc(L, x, 3)
    torch.cuda.synchronize()
    assert torch.equal(gs.cpu(), rs.cpu())
    assert torch.equal(gc, rc)
    del x, rc, gc
    torch.cuda.empty_cache()
