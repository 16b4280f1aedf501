"""The decode GEMM (tcgen05, swapped operands, split-K with an on-GPU reduction) against fp32."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ext():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from pdattention_b200.ops._ext import require

    return require()


@pytest.mark.parametrize("m,n,k,splits", [(64, 4096, 512, 0), (1, 256, 64, 0), (17, 1000, 4096, 0),
                                          (64, 1792, 4096, 8), (40, 384, 1024, 1), (64, 16032, 4096, 0)])
def test_matches_fp32(ext, m, n, k, splits):
    gen = torch.Generator(device="cuda").manual_seed(m * 7 + n)
    x = torch.randn(m, k, device="cuda", generator=gen).bfloat16()
    w = (torch.randn(n, k, device="cuda", generator=gen) * 0.05).bfloat16()
    bias = torch.randn(n, device="cuda", generator=gen).bfloat16()
    res = torch.randn(m, n, device="cuda", generator=gen).bfloat16()
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    for _ in range(2):  # the split-K workspace and counters are reused: a second call must agree
        ext.decode_gemm(x, w, bias, res, out, None, 0, splits, [], [], 0, None, 0, None)
        want = x.float() @ w.float().t() + bias.float() + res.float()
        torch.cuda.synchronize()
        err = (out.float() - want).abs().max().item()
        assert err <= 2e-2 * want.abs().max().item(), (m, n, k, splits, err)


def test_two_outputs_and_strided_input(ext):
    """Columns past split_col (the routing-query rows of a QKV weight) land in the second output."""
    gen = torch.Generator(device="cuda").manual_seed(3)
    m, k, n, split = 64, 1024, 768 + 512, 768
    base = torch.randn(m, k + 64, device="cuda", generator=gen).bfloat16()
    x = base[:, :k]  # row stride k + 64
    w = (torch.randn(n, k, device="cuda", generator=gen) * 0.05).bfloat16()
    out = torch.empty(m, split, device="cuda", dtype=torch.bfloat16)
    out2 = torch.empty(m, n - split, device="cuda", dtype=torch.bfloat16)
    ext.decode_gemm(x, w, None, None, out, out2, split, 0, [], [], 0, None, 0, None)
    want = x.float() @ w.float().t()
    torch.cuda.synchronize()
    scale = want.abs().max().item()
    assert (out.float() - want[:, :split]).abs().max().item() <= 2e-2 * scale
    assert (out2.float() - want[:, split:]).abs().max().item() <= 2e-2 * scale
