"""The allocation-free column-sum entry point, called through its exported C symbol.

``pra_colsum_noalloc`` is for callers that cannot allocate device memory where
they call it: hosts that reserve all device memory up front, or code running
where its host forbids calls that can synchronise the device (cudaMalloc can).
It must give the same column sums as the library's ordinary op and as an fp32
``torch.sum``, on consecutive calls that reuse its fixed scratch array; it must
accept a shape that fills that array exactly and refuse one that would overflow
it or that hands it a misaligned matrix.  This file sorts last so a run that
stops at the first failure has already run every other test.
"""

import ctypes

import pytest
import torch


def _load():
    from pdattention_b200.ops import _ext

    so = _ext._so_path()
    if so is None:
        pytest.skip("extension not built")
    handle = ctypes.CDLL(str(so))
    fn = handle.pra_colsum_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    handle.pra_colsum_noalloc_capacity.restype = ctypes.c_longlong
    return handle


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from pdattention_b200.ops import _ext

    _ext.require()
    return _load()


def _call(lib, g: torch.Tensor, out: torch.Tensor) -> int:
    stream = torch.cuda.current_stream().cuda_stream
    return lib.pra_colsum_noalloc(ctypes.c_void_p(g.data_ptr()), g.shape[0], g.shape[1],
                                  ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(stream))


def _check(out: torch.Tensor, g: torch.Tensor) -> None:
    expected = g.float().sum(dim=0)
    err = (out.float() - expected).abs().max().item()
    scale = expected.abs().max().item() + 1e-6
    assert err <= 2e-2 * scale, (tuple(g.shape), err, scale)


@pytest.mark.gpu
def test_matches_fp32_sum_and_existing_colsum_on_consecutive_calls(lib):
    from pdattention_b200.ops._ext import require

    ext = require()
    for seed, (m, n) in enumerate([(6144, 3072), (777, 768)]):
        gen = torch.Generator(device="cuda").manual_seed(seed)
        g = torch.randn(m, n, device="cuda", generator=gen).bfloat16()
        out = torch.empty(n, device="cuda", dtype=torch.bfloat16)
        assert _call(lib, g, out) == 0
        torch.cuda.synchronize()
        _check(out, g)
        expected = ext.colsum(g)
        assert torch.equal(out, expected), (m, n)  # same kernels, same order of summation


@pytest.mark.gpu
def test_captured_in_a_cuda_graph_and_replayed_on_new_data(lib):
    """The use it exists for: after one warm-up call (which looks up the scratch address), a call
    made while a CUDA graph is being captured launches kernels only, and replays of that graph
    sum whatever the input buffer holds at replay time."""
    m, n = 2048, 1536
    g = torch.randn(m, n, device="cuda").bfloat16()
    out = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    assert _call(lib, g, out) == 0  # warm-up outside the capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        rc = _call(lib, g, out)
    assert rc == 0
    for seed in (1, 2):
        g.copy_(torch.randn(m, n, device="cuda", generator=torch.Generator(device="cuda").manual_seed(seed)))
        graph.replay()
        torch.cuda.synchronize()
        _check(out, g)


@pytest.mark.gpu
def test_accepts_a_shape_that_fills_the_scratch_exactly(lib):
    capacity = lib.pra_colsum_noalloc_capacity()
    m, n = 16384, 4096  # 256 partial rows x 4096 columns
    assert 256 * n == capacity
    g = torch.randn(m, n, device="cuda", generator=torch.Generator(device="cuda").manual_seed(7)).bfloat16()
    out = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    assert _call(lib, g, out) == 0
    torch.cuda.synchronize()
    _check(out, g)


@pytest.mark.gpu
def test_rejects_shapes_beyond_the_scratch_capacity(lib):
    capacity = lib.pra_colsum_noalloc_capacity()
    m, n = 8192, 8200  # 128 partial rows x 8200 columns > capacity
    assert 128 * n > capacity
    g = torch.zeros(m, n, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    assert _call(lib, g, out) != 0


def test_rejects_misaligned_input_before_touching_the_device():
    """A bf16 view starting at an odd element is refused with an error code, not launched."""
    lib = _load()
    rc = lib.pra_colsum_noalloc(ctypes.c_void_p(0x10002), 4, 8, ctypes.c_void_p(0x20000), ctypes.c_void_p(0))
    assert rc != 0
    rc = lib.pra_colsum_noalloc(ctypes.c_void_p(0x10000), 4, 7, ctypes.c_void_p(0x20000), ctypes.c_void_p(0))
    assert rc != 0  # odd N
