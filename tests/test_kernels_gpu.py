"""sm_100a kernels against fp32 PyTorch restatements of the same math (GPU only)."""

import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ext():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from pdattention_b200.ops._ext import require

    return require()


def _bf(*shape, scale=1.0, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, device="cuda", generator=g) * scale).bfloat16()


def _close(a, b, tol):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    ref = b.abs().max().item() + 1e-6
    assert err <= tol * ref, f"max err {err} vs ref scale {ref}"


@pytest.mark.parametrize("m,n,k", [(300, 256, 192), (2048, 768, 768), (520, 3072, 768), (8192, 2304, 768)])
def test_stream_k_gemms(ext, m, n, k):
    """The stream-K GEMM instantiations against fp32, including ragged M."""
    a, w = _bf(m, k, seed=11), _bf(n, k, scale=0.05, seed=12)
    dy = _bf(m, n, seed=15)
    dx = torch.empty(m, k, device="cuda", dtype=torch.bfloat16)
    for kind in ("nn_sk",):
        ext.gemm(kind, dy, w, None, dx, None, None, 1.0, 0.0, None)
        _close(dx, dy.float() @ w.float(), 2e-2)
    gw = torch.empty(n, k, device="cuda", dtype=torch.bfloat16)
    for kind in ("wgrad_sk",):
        ext.gemm(kind, dy, a, None, gw, None, None, 1.0, 0.0, None)
        _close(gw, dy.float().T @ a.float(), 2e-2)


@pytest.mark.parametrize("m,n,k", [(300, 256, 192), (2048, 768, 768), (96, 3072, 768)])
def test_gemm_variants(ext, m, n, k):
    a, w, bias, res = _bf(m, k, seed=1), _bf(n, k, scale=0.05, seed=2), _bf(n, seed=3), _bf(m, n, seed=4)
    d = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    ext.gemm("tn", a, w, res, d, bias, None, 1.0, 1.0, None)
    _close(d, a.float() @ w.float().T + bias.float() + res.float(), 2e-2)
    z = torch.empty_like(d)
    ext.gemm("tn_gelu", a, w, None, d, bias, z, 1.0, 0.0, None)
    zr = a.float() @ w.float().T + bias.float()
    _close(z, zr, 2e-2)
    _close(d, F.gelu(zr), 2e-2)
    dy = _bf(m, n, seed=5)
    dx = torch.empty(m, k, device="cuda", dtype=torch.bfloat16)
    ext.gemm("nn", dy, w, None, dx, None, None, 1.0, 0.0, None)
    _close(dx, dy.float() @ w.float(), 2e-2)
    # fused GELU derivative: dz = gelu'(z) * (dy2 @ w2) with w2 [n2=k?]
    w2 = _bf(n, n, scale=0.05, seed=6)
    dz = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    ext.gemm("nn_dgelu", dy, w2, None, dz, None, z, 1.0, 0.0, None)
    zf = z.float().requires_grad_(True)
    F.gelu(zf).backward(dy.float() @ w2.float())
    _close(dz, zf.grad, 3e-2)
    gw = torch.empty(n, k, device="cuda", dtype=torch.bfloat16)
    ext.gemm("wgrad", dy, a, None, gw, None, None, 1.0, 0.0, None)
    _close(gw, dy.float().T @ a.float(), 2e-2)
    scale = torch.tensor([0.5], device="cuda")
    ext.gemm("wgrad", dy, a, gw.clone(), gw, None, None, 1.0, 1.0, scale)
    _close(gw, 1.5 * (dy.float().T @ a.float()), 2e-2)


def test_epilogue_gelu_matches_erf_gelu(ext):
    """The GEMM epilogues' GELU (Abramowitz & Stegun 7.1.26 erf) and its derivative against
    fp32 PyTorch erf GELU over [-12, 12]: the formula's 1.5e-7 bound plus fp32 rounding."""
    z = torch.cat([torch.linspace(-12, 12, 200001, device="cuda"), torch.randn(100000, device="cuda") * 3])
    y, dy = ext.gelu_probe(z.contiguous())
    zd = z.double().requires_grad_(True)
    ref = torch.nn.functional.gelu(zd)
    ref.backward(torch.ones_like(zd))
    err = (y.double() - ref.detach()).abs() / (1 + zd.detach().abs())
    derr = (dy.double() - zd.grad).abs()
    assert err.max() < 2e-6, float(err.max())
    assert derr.max() < 2e-6, float(derr.max())


@pytest.mark.parametrize("rms", [False, True])
def test_norm(ext, rms):
    x, w, b = _bf(513, 768, seed=1), _bf(768, seed=2), _bf(768, seed=3)
    y, mean, rstd = ext.norm_fwd(x, w, None if rms else b, 1e-5, rms)
    xf = x.float().requires_grad_(True)
    if rms:
        ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5) * w.float()
    else:
        ref = F.layer_norm(xf, (768,), w.float(), b.float(), 1e-5)
    _close(y, ref, 2e-2)
    dy = _bf(513, 768, seed=4)
    dx, dw, db = ext.norm_bwd(dy, x, w, mean, rstd, None, rms)
    wf = w.float().requires_grad_(True)
    bf = b.float().requires_grad_(True)
    xf2 = x.float().requires_grad_(True)
    if rms:
        out = xf2 * torch.rsqrt(xf2.pow(2).mean(-1, keepdim=True) + 1e-5) * wf
    else:
        out = F.layer_norm(xf2, (768,), wf, bf, 1e-5)
    out.backward(dy.float())
    _close(dx, xf2.grad, 3e-2)
    _close(dw, wf.grad, 3e-2)
    if not rms:
        _close(db, bf.grad, 3e-2)


def _attention_reference(q, k, v, mem_k, mem_v, key_valid, scale):
    """fp32 per-row restatement: [memory (all visible) ; local causal + padding]."""
    b, t, h, d = q.shape
    out = torch.zeros(b, t, h, d, device=q.device)
    for row in range(b):
        mk = mem_k[row] if mem_k is not None else q.new_zeros(0, h, d)
        mv = mem_v[row] if mem_v is not None else q.new_zeros(0, h, d)
        keys = torch.cat([mk, k[row]], 0).float()
        vals = torch.cat([mv, v[row]], 0).float()
        s = torch.einsum("thd,shd->hts", q[row].float(), keys) * scale
        m = mk.shape[0]
        vis = torch.ones(t, m + t, dtype=torch.bool, device=q.device)
        vis[:, m:] = torch.ones(t, t, dtype=torch.bool, device=q.device).tril()
        if key_valid is not None:
            vis[:, m:] &= key_valid[row].bool()[None, :]
        s = s.masked_fill(~vis[None], float("-inf"))
        p = torch.softmax(s, -1).nan_to_num(0.0)
        out[row] = torch.einsum("hts,shd->thd", p, vals)
    return out


@pytest.mark.parametrize("head_dim", [32, 64, 128])
@pytest.mark.parametrize("with_memory", [False, True])
def test_attention_fwd_bwd(ext, head_dim, with_memory):
    torch.manual_seed(0)
    b, t, h = 3, 150, 4
    d = h * head_dim
    qkv = _bf(b, t, 3 * d, seed=1)
    key_valid = torch.ones(b, t, dtype=torch.uint8, device="cuda")
    key_valid[1, 100:] = 0
    scale = 1.0 / math.sqrt(head_dim)
    memory = None
    mem_lists = None
    if with_memory:
        pool = _bf(500, 3 * d, seed=7)
        lens = [70, 0, 131]
        idx = torch.zeros(b, 140, dtype=torch.int32, device="cuda")
        mem_lists = []
        for r, n in enumerate(lens):
            rows = torch.randperm(500, device="cuda")[:n].int()
            idx[r, :n] = rows
            mem_lists.append(rows.long())
        from pdattention_b200.ops.kernels import MemoryView

        memory = MemoryView(pool[:, d:2 * d], pool[:, 2 * d:], idx, torch.tensor(lens, dtype=torch.int32,
                                                                                  device="cuda"))
    from pdattention_b200.ops.kernels import attention

    x = qkv.clone().requires_grad_(True)
    out = attention(x, h, head_dim, memory, key_valid, scale)
    q = qkv[..., :d].view(b, t, h, head_dim)
    k = qkv[..., d:2 * d].view(b, t, h, head_dim)
    v = qkv[..., 2 * d:].view(b, t, h, head_dim)
    mk = mv = None
    if with_memory:
        mk = [pool[rows, d:2 * d].view(-1, h, head_dim) for rows in mem_lists]
        mv = [pool[rows, 2 * d:].view(-1, h, head_dim) for rows in mem_lists]
    qf = q.float().requires_grad_(True)
    kf = k.float().requires_grad_(True)
    vf = v.float().requires_grad_(True)
    ref = _attention_reference(qf, kf, vf, mk, mv, key_valid, scale)
    _close(out.view(b, t, h, head_dim), ref, 2e-2)
    dout = _bf(b, t, d, seed=9)
    out.backward(dout)
    ref.backward(dout.float().view(b, t, h, head_dim))
    g = x.grad.view(b, t, 3, h, head_dim)
    _close(g[:, :, 0], qf.grad, 3e-2)
    _close(g[:, :, 1], kf.grad, 3e-2)
    _close(g[:, :, 2], vf.grad, 3e-2)


def test_cross_entropy_and_head(ext):
    from pdattention_b200.ops.kernels import WeightSlot, lm_head_loss

    m, dmodel, vocab, vpad = 777, 256, 1000, 1024
    hidden = _bf(m, dmodel, seed=1).requires_grad_(True)
    w = torch.zeros(vpad, dmodel, device="cuda", dtype=torch.bfloat16)
    w[:vocab] = _bf(vocab, dmodel, scale=0.05, seed=2)
    gw = torch.zeros_like(w)
    labels = torch.randint(0, vocab, (m,), device="cuda")
    labels[::7] = 0
    loss = lm_head_loss(hidden, WeightSlot(w=w, gw=gw), labels, vocab, 0)
    hf = hidden.detach().float().requires_grad_(True)
    wf = w[:vocab].float().requires_grad_(True)
    ref = F.cross_entropy(hf @ wf.T, labels, ignore_index=0)
    assert abs(loss.item() - ref.item()) < 2e-2 * max(1.0, abs(ref.item()))
    loss.backward()
    ref.backward()
    _close(hidden.grad, hf.grad, 5e-2)
    _close(gw[:vocab], wf.grad, 5e-2)
    assert gw[vocab:].abs().max().item() == 0.0


def test_adamw_matches_torch(ext):
    n = 10000
    p0 = torch.randn(n, device="cuda")
    grads = [torch.randn(n, device="cuda") * 3 for _ in range(3)]
    ref = p0.clone().requires_grad_(True)
    opt = torch.optim.AdamW([ref], lr=1e-3, weight_decay=0.01)
    mine, m, v = p0.clone(), torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    shadow = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    for step, g in enumerate(grads, start=1):
        ref.grad = g.clone()
        torch.nn.utils.clip_grad_norm_([ref], 1.0)
        opt.step()
        norm, coef = ext.grad_norm(g, 1.0)
        assert abs(norm.item() - g.norm().item()) < 1e-3 * g.norm().item()
        ext.adamw(mine, shadow, g, m, v, 1e-3, 0.9, 0.999, 1e-8, 0.01, step, coef, 1.0)
    assert torch.allclose(mine, ref.detach(), atol=1e-5)
    assert torch.allclose(shadow.float(), mine, atol=1e-2)


def test_gist_mean_and_kmeans_match_strategies(ext):
    from types import SimpleNamespace

    from pdattention_b200.config import PRAConfig
    from pdattention_b200.memory.gists import compute_gists, kmeanspp_random_stream

    d = 96
    lens = [64, 64, 37, 5]
    starts = [0, 64, 128, 192]
    pool = _bf(256, 2 * d, seed=3)
    pk, pv = pool[:, :d], pool[:, d:]
    start = torch.tensor(starts, dtype=torch.int32, device="cuda")
    length = torch.tensor(lens, dtype=torch.int32, device="cuda")
    gk, gv, gn = ext.gist_mean(pk, pv, start, length)
    for c, (s, n) in enumerate(zip(starts, lens)):
        assert torch.allclose(gk[c], pk[s:s + n].float().mean(0), atol=1e-4)
        assert torch.allclose(gn[c], F.normalize(pk[s:s + n].float().mean(0), dim=0), atol=1e-4)
    cfg = PRAConfig()
    firsts, draws, offs, flat = [], [], [], 0
    for n in lens:
        first, exp = kmeanspp_random_stream(n, 2, cfg.gist_kmeans_seed)
        firsts.append(first)
        offs.append(flat)
        draws.append(exp.flatten())
        flat += exp.numel()
    out = ext.gist_kmeans(pk, pv, start, length, 2, cfg.gist_kmeans_max_iters, cfg.gist_kmeans_tol, True, True, True,
                          torch.tensor(firsts, dtype=torch.int32, device="cuda"),
                          torch.zeros(1, dtype=torch.int32, device="cuda"), torch.cat(draws).cuda(),
                          torch.tensor(offs, dtype=torch.int32, device="cuda"))
    gk2, gv2, count = out[0], out[1], out[2]
    ctx = SimpleNamespace(level="chunk", token_ids=(), tokenizer=None, ref_end_token="", gru_pooler=None)
    for c, (s, n) in enumerate(zip(starts, lens)):
        ref = compute_gists(keys=pk[s:s + n].float().cpu(), values=pv[s:s + n].float().cpu(), mode="kmeans",
                            num_gists=2, config=cfg, context=ctx)
        assert int(count[c]) == ref.k.shape[0]
        assert torch.allclose(gk2[c, : ref.k.shape[0]].cpu(), ref.k, atol=2e-3)
        assert torch.allclose(gv2[c, : ref.v.shape[0]].cpu(), ref.v, atol=2e-3)


def test_route_kernel_matches_object_search(ext):
    """Device routing + budget + materialisation equals the host object path on random namespaces."""
    from pdattention_b200.models.fastpath import routing_selftest

    routing_selftest(torch.device("cuda"))


def _gqa_reference(q, k, v, mem_k, mem_v, key_valid, scale, kv_heads):
    """fp32 restatement with grouped KV heads: q [B,T,H,D], k/v [B,T,Hkv,D], memory per row."""
    h = q.shape[2]
    rep = h // kv_heads
    expand = (lambda x: x.repeat_interleave(rep, dim=-2) if x is not None else None)
    mk = [expand(m) for m in mem_k] if mem_k is not None else None
    mv = [expand(m) for m in mem_v] if mem_v is not None else None
    return _attention_reference(q, expand(k), expand(v), mk, mv, key_valid, scale)


@pytest.mark.parametrize("head_dim", [64, 128])
@pytest.mark.parametrize("t,lens,logit_scale", [(300, [260, 513], 1.0), (300, [0, 129], 6.0), (1, [64, 0], 1.0),
                                                (1024, [0, 0], 3.0), (64, [200, 0], 1.0), (37, [70, 129], 6.0),
                                                (64, [1000, 3], 2.0)])
def test_attention_fwd_tcgen05(ext, head_dim, t, lens, logit_scale):
    """The tcgen05 forward against fp32 PyTorch and the mma.sync forward: GQA (8 heads over 2),
    memory blocks gathered from a pool, padding masks, and logits large enough that the lazily
    raised running maximum rescales O in TMEM."""
    b, h, hkv = 2, 8, 2
    d, dk = h * head_dim, hkv * head_dim
    q = _bf(b, t, d, seed=11)
    k = _bf(b, t, dk, seed=12)
    v = _bf(b, t, dk, seed=13)
    key_valid = torch.ones(b, t, dtype=torch.uint8, device="cuda")
    if t > 10:
        key_valid[0, t // 3: t // 2] = 0
    pool = _bf(1200, 2 * dk, seed=14)
    g = torch.Generator(device="cuda").manual_seed(15)
    idx = torch.zeros(b, max(max(lens), 1), dtype=torch.int32, device="cuda")
    rows = []
    for r, n in enumerate(lens):
        sel = torch.randperm(1200, device="cuda", generator=g)[:n].int()
        idx[r, :n] = sel
        rows.append(sel.long())
    mem_len = torch.tensor(lens, dtype=torch.int32, device="cuda")
    scale = logit_scale / math.sqrt(head_dim)
    status = ext.attention_status(0)
    status.zero_()
    outs = {}
    for impl in ("tcgen05", "mma"):
        ext.set_attention_impl(impl)
        outs[impl] = ext.attention_fwd(q, k, v, h, hkv, head_dim, pool[:, :dk], pool[:, dk:], idx, mem_len,
                                       key_valid, scale)
    ext.set_attention_impl("tcgen05")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    mk = [pool[r_, :dk].view(-1, hkv, head_dim) for r_ in rows]
    mv = [pool[r_, dk:].view(-1, hkv, head_dim) for r_ in rows]
    ref = _gqa_reference(q.view(b, t, h, head_dim), k.view(b, t, hkv, head_dim), v.view(b, t, hkv, head_dim),
                         mk, mv, key_valid, scale, hkv)
    out_tc, lse_tc = outs["tcgen05"]
    out_mma, lse_mma = outs["mma"]
    _close(out_tc.view(b, t, h, head_dim), ref, 2e-2)
    _close(out_tc, out_mma, 2e-2)
    finite = torch.isfinite(lse_mma)
    assert torch.equal(finite, torch.isfinite(lse_tc))
    assert (lse_tc[finite] - lse_mma[finite]).abs().max().item() < 1e-2 * max(1.0, lse_mma[finite].abs().max().item())


@pytest.mark.parametrize("t,lens,logit_scale", [(300, [260, 513], 1.0), (1024, [0, 64], 4.0), (97, [5, 0], 1.0)])
def test_attention_bwd_tcgen05(ext, t, lens, logit_scale):
    """dQ, dK, dV from the tcgen05 backward against fp32 autograd and the mma.sync backward
    (head dim 64, memory keys, padding mask)."""
    b, h, hd = 2, 4, 64
    d = h * hd
    qkv = _bf(b, t, 3 * d, seed=21)
    q, k, v = qkv[..., :d], qkv[..., d:2 * d], qkv[..., 2 * d:]
    key_valid = torch.ones(b, t, dtype=torch.uint8, device="cuda")
    key_valid[1, t // 4: t // 3] = 0
    pool = _bf(1200, 2 * d, seed=22)
    g = torch.Generator(device="cuda").manual_seed(23)
    idx = torch.zeros(b, max(lens), dtype=torch.int32, device="cuda")
    rows = []
    for r, n in enumerate(lens):
        sel = torch.randperm(1200, device="cuda", generator=g)[:n].int()
        idx[r, :n] = sel
        rows.append(sel.long())
    mem_len = torch.tensor(lens, dtype=torch.int32, device="cuda")
    scale = logit_scale / math.sqrt(hd)
    out, lse = ext.attention_fwd(q, k, v, h, h, hd, pool[:, :d], pool[:, d:], idx, mem_len, key_valid, scale)
    dout = _bf(b, t, d, seed=24)
    status = ext.attention_status(0)
    status.zero_()
    grads = {}
    for impl in ("tcgen05", "mma"):
        ext.set_attention_impl(impl)
        (grads[impl],) = ext.attention_bwd(dout, q, k, v, out, lse, h, hd, pool[:, :d], pool[:, d:], idx, mem_len,
                                           key_valid, scale)
    ext.set_attention_impl("tcgen05")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    g_tc = grads["tcgen05"].view(b, t, 3, h, hd)
    g_mma = grads["mma"].view(b, t, 3, h, hd)
    for i in range(3):
        _close(g_tc[:, :, i], g_mma[:, :, i], 2e-2)
    qf = q.float().view(b, t, h, hd).requires_grad_(True)
    kf = k.float().view(b, t, h, hd).requires_grad_(True)
    vf = v.float().view(b, t, h, hd).requires_grad_(True)
    mk = [pool[r_, :d].view(-1, h, hd) for r_ in rows]
    mv = [pool[r_, d:].view(-1, h, hd) for r_ in rows]
    ref = _attention_reference(qf, kf, vf, mk, mv, key_valid, scale)
    ref.backward(dout.float().view(b, t, h, hd))
    _close(g_tc[:, :, 0], qf.grad, 3e-2)
    _close(g_tc[:, :, 1], kf.grad, 3e-2)
    _close(g_tc[:, :, 2], vf.grad, 3e-2)


def test_attention_fwd_packed_odd_batch(ext):
    """Sequences of <= 64 tokens run two per tcgen05 tile; an odd batch leaves the last tile
    half empty."""
    b, t, h, hd = 3, 50, 4, 64
    d = h * hd
    q, k, v = _bf(b, t, d, seed=31), _bf(b, t, d, seed=32), _bf(b, t, d, seed=33)
    key_valid = torch.ones(b, t, dtype=torch.uint8, device="cuda")
    key_valid[2, 10:20] = 0
    pool = _bf(300, 2 * d, seed=34)
    lens = [65, 0, 130]
    idx = torch.zeros(b, 130, dtype=torch.int32, device="cuda")
    rows = []
    for r, n in enumerate(lens):
        sel = torch.randperm(300, device="cuda")[:n].int()
        idx[r, :n] = sel
        rows.append(sel.long())
    mem_len = torch.tensor(lens, dtype=torch.int32, device="cuda")
    scale = 1.0 / math.sqrt(hd)
    out, lse = ext.attention_fwd(q, k, v, h, h, hd, pool[:, :d], pool[:, d:], idx, mem_len, key_valid, scale)
    mk = [pool[r_, :d].view(-1, h, hd) for r_ in rows]
    mv = [pool[r_, d:].view(-1, h, hd) for r_ in rows]
    ref = _attention_reference(q.view(b, t, h, hd), k.view(b, t, h, hd), v.view(b, t, h, hd), mk, mv, key_valid,
                               scale)
    _close(out.view(b, t, h, hd), ref, 2e-2)
    ext.set_attention_impl("mma")
    _, lse_mma = ext.attention_fwd(q, k, v, h, h, hd, pool[:, :d], pool[:, d:], idx, mem_len, key_valid, scale)
    ext.set_attention_impl("tcgen05")
    assert (lse - lse_mma).abs().max().item() < 1e-2
