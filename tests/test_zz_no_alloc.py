"""The allocation-free column-sum entry point, called through its exported C symbol.

``pra_colsum_noalloc`` is for callers that cannot allocate device memory where
they call it (hosts that reserve all memory up front, or code issued during
CUDA-graph capture where cudaMalloc is illegal).  It must give the same result
as the library's ordinary column-sum op, on consecutive calls that reuse its
fixed scratch array, and must refuse shapes that would overflow that array.
This file sorts last so a run that stops at the first failure has already run
every other test.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from pdattention_b200.ops import _ext

    _ext.require()
    so = _ext._so_path()
    assert so is not None, "extension not built"
    handle = ctypes.CDLL(str(so))
    fn = handle.pra_colsum_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    handle.pra_colsum_noalloc_capacity.restype = ctypes.c_longlong
    return handle


def _call(lib, g: torch.Tensor, out: torch.Tensor) -> int:
    stream = torch.cuda.current_stream().cuda_stream
    return lib.pra_colsum_noalloc(ctypes.c_void_p(g.data_ptr()), g.shape[0], g.shape[1],
                                  ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(stream))


def test_matches_existing_colsum_on_consecutive_calls(lib):
    from pdattention_b200.ops._ext import require

    ext = require()
    for seed, (m, n) in enumerate([(6144, 3072), (777, 768)]):
        gen = torch.Generator(device="cuda").manual_seed(seed)
        g = torch.randn(m, n, device="cuda", generator=gen).bfloat16()
        out = torch.empty(n, device="cuda", dtype=torch.bfloat16)
        assert _call(lib, g, out) == 0
        expected = ext.colsum(g)
        torch.cuda.synchronize()
        err = (out.float() - expected.float()).abs().max().item()
        scale = expected.float().abs().max().item() + 1e-6
        assert err <= 2e-2 * scale, (m, n, err, scale)


def test_rejects_shapes_beyond_the_scratch_capacity(lib):
    capacity = lib.pra_colsum_noalloc_capacity()
    m, n = 8192, 8200  # 128 partial rows x 8200 columns > capacity
    assert 128 * n > capacity
    g = torch.zeros(m, n, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    assert _call(lib, g, out) != 0
