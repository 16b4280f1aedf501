"""The decode GEMM (tcgen05, swapped operands, split-K reduced across a thread-block cluster in
distributed shared memory) against fp32."""

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
    for _ in range(2):  # a second call (same tensor maps, same launch) must agree
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


@pytest.mark.parametrize("head_dim,heads,kv_heads,bias", [(128, 4, 2, False), (64, 8, 4, True)])
def test_rotary_qkv_epilogue_matches_gemm_then_rope(ext, head_dim, heads, kv_heads, bias):
    """One decode GEMM writes rotated q, rotated k / plain v into their cache rows and the
    routing-query columns, as the QKV GEMM followed by the rotary copies does."""
    gen = torch.Generator(device="cuda").manual_seed(head_dim)
    m, k = 24, 512
    qd, kd, rd = heads * head_dim, kv_heads * head_dim, 256
    n = qd + 2 * kd + rd
    x = torch.randn(m, k, device="cuda", generator=gen).bfloat16()
    w = (torch.randn(n, k, device="cuda", generator=gen) * 0.05).bfloat16()
    b = torch.randn(n, device="cuda", generator=gen).bfloat16() if bias else None
    half = head_dim // 2
    inv = 1.0 / (10000.0 ** (torch.arange(half, dtype=torch.float64) / half))
    ang = torch.arange(4096, dtype=torch.float64)[:, None] * inv[None]
    cos, sin = ang.cos().float().cuda(), ang.sin().float().cuda()
    pos = torch.randint(0, 4000, (m,), device="cuda", generator=gen, dtype=torch.int32)
    rows = (torch.arange(m, device="cuda", dtype=torch.int32) * 7 + 3).int()
    caches = [torch.zeros(m * 7 + 8, kd, device="cuda", dtype=torch.bfloat16) for _ in range(4)]
    q_fused, q_ref = (torch.empty(m, qd, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    r_fused = torch.empty(m, rd, device="cuda", dtype=torch.bfloat16)
    ext.decode_qkv_rope(x, w, b, q_fused, caches[0], caches[1], rows, pos, cos, sin, head_dim, qd, qd + kd,
                        qd + 2 * kd, r_fused)
    full = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    ext.gemm("tn", x, w, None, full, b, None, 1.0, 0.0, None)
    ext.rope_copy(full[:, qd: qd + kd], caches[2], rows, pos, cos, sin, kv_heads, head_dim)
    ext.rope_copy(full[:, qd + kd: qd + 2 * kd], caches[3], rows, None, None, None, kv_heads, head_dim)
    ext.rope_copy(full[:, :qd], q_ref, None, pos, cos, sin, heads, head_dim)
    torch.cuda.synchronize()

    def close(a, r):
        scale = r.float().abs().max().item() + 1e-6
        return (a.float() - r.float()).abs().max().item() <= 2e-2 * scale

    assert close(q_fused, q_ref)
    assert close(caches[0], caches[2]) and close(caches[1], caches[3])
    assert close(r_fused, full[:, qd + 2 * kd:])


@pytest.mark.parametrize("m,n,k", [(64, 4096, 1024), (3, 512, 1024), (64, 2048, 128)])
def test_fp32_scores_output(ext, m, n, k):
    """fp32 output (the routing scores; 2-stage ring) against the fp32 product."""
    gen = torch.Generator(device="cuda").manual_seed(n + k)
    x = torch.randn(m, k, device="cuda", generator=gen).bfloat16()
    w = torch.nn.functional.normalize(torch.randn(n, k, device="cuda", generator=gen), dim=-1).bfloat16()
    out = torch.full((m, n), float("nan"), device="cuda")
    ext.decode_gemm(x, w, None, None, out, None, 0, 0, [], [], 0, None, 0, None)
    want = x.float() @ w.float().t()
    assert torch.allclose(out, want, atol=1e-3, rtol=1e-3), (out - want).abs().max()


def test_resident_cluster_counts(ext):
    """How many split-K clusters can be resident at once (the fused all-reduce lowers its split
    count until its grid fits): an unsplit 32-tile row-parallel grid always fits, and wider
    clusters never fit more."""
    counts = [ext.decode_gemm_resident_clusters(s) for s in (1, 2, 4, 8)]
    print("resident clusters for 1/2/4/8 splits:", counts)
    assert counts[0] >= 32
    assert all(a >= b for a, b in zip(counts, counts[1:])), counts


@pytest.mark.parametrize("m,f,k", [(64, 1792, 4096), (5, 256, 128)])
def test_swiglu_epilogue_matches_gemm_then_silu(ext, m, f, k):
    """A [gate | up]-interleaved weight (runs of 64) with the SwiGLU epilogue equals fp32
    silu(x G^T) * (x U^T); the blocked silu_mul on the GEMM's output agrees."""
    gen = torch.Generator(device="cuda").manual_seed(f + k)
    x = torch.randn(m, k, device="cuda", generator=gen).bfloat16()
    gate = (torch.randn(f, k, device="cuda", generator=gen) * 0.05).bfloat16()
    up = (torch.randn(f, k, device="cuda", generator=gen) * 0.05).bfloat16()
    blocked = torch.stack([gate.view(f // 64, 64, k), up.view(f // 64, 64, k)], 1).reshape(2 * f, k).contiguous()
    act = torch.empty(m, f, device="cuda", dtype=torch.bfloat16)
    ext.decode_gemm(x, blocked, None, None, act, None, 0, 0, [], [], 0, None, 0, None, swiglu=True)
    g, u = x.float() @ gate.float().t(), x.float() @ up.float().t()
    want = torch.nn.functional.silu(g) * u
    assert torch.allclose(act.float(), want, atol=2e-2 * want.abs().max().item(), rtol=2e-2)
    gu = torch.empty(m, 2 * f, device="cuda", dtype=torch.bfloat16)
    ext.decode_gemm(x, blocked, None, None, gu, None, 0, 0, [], [], 0, None, 0, None)
    act2 = torch.empty_like(act)
    ext.silu_mul(gu, act2, 64)
    assert torch.allclose(act2.float(), want, atol=2e-2 * want.abs().max().item(), rtol=2e-2)


def test_folded_rmsnorm_producer_and_consumer(ext):
    """A producer GEMM (with residual) writes per-tile row sums of squares of its bf16 output; a
    consumer GEMM whose weight carries the norm weight scales its rows by rsqrt(mean square + eps):
    equal to RMSNorm then GEMM in fp32."""
    gen = torch.Generator(device="cuda").manual_seed(21)
    m, d, k, n, eps = 37, 1024, 512, 768, 1e-5
    a = torch.randn(m, k, device="cuda", generator=gen).bfloat16()
    wo = (torch.randn(d, k, device="cuda", generator=gen) * 0.05).bfloat16()
    res = torch.randn(m, d, device="cuda", generator=gen).bfloat16()
    x = torch.empty(m, d, device="cuda", dtype=torch.bfloat16)
    ss = torch.full((d // 128, 64), float("nan"), device="cuda")
    ext.decode_gemm(a, wo, None, res, x, None, 0, 0, [], [], 0, None, 0, None, ss_out=ss)
    want_ss = (x.float() ** 2).view(m, d // 128, 128).sum(-1).t()
    assert torch.allclose(ss[:, :m], want_ss, rtol=1e-5, atol=1e-3)
    g = (1 + 0.1 * torch.randn(d, device="cuda", generator=gen)).bfloat16()
    w = (torch.randn(n, d, device="cuda", generator=gen) * 0.05).bfloat16()
    wg = (w.float() * g.float()[None]).bfloat16()
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    ext.decode_gemm(x, wg, None, None, out, None, 0, 0, [], [], 0, None, 0, None, ss_in=ss, ss_tiles=d // 128,
                    ss_dim=d, ss_eps=eps)
    xf = x.float()
    h = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * g.float()
    want = h @ w.float().t()
    assert torch.allclose(out.float(), want, atol=2e-2 * want.abs().max().item(), rtol=2e-2)
