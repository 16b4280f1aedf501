"""Counter-based dropout kernels and the vanilla / mixed blocks on the device path.

The oracle of the masks is a NumPy restatement of Philox4x32-10 (Salmon et al., SC 2011)
over the same (seed, offset, element) stream; attention with dropout is checked
against an fp32 PyTorch restatement that applies that mask to the softmax
probabilities (forward, and the gradients through torch autograd).  The vanilla and
mixed blocks are checked against the fp32 object path in eval mode.
"""

import copy
import math
from pathlib import Path

import numpy as np
import pytest
import torch

from pdattention_b200.config import ResolverServiceConfig, TrainConfig
from pdattention_b200.models import TinyPRAModel
from pdattention_b200.models.fastpath import attach_device_runtime
from pdattention_b200.pra_train import _pra_batch_step
from pdattention_b200.smoke import tiny_batch, tiny_config

pytestmark = pytest.mark.gpu
M32 = np.uint64(0xFFFFFFFF)


@pytest.fixture(scope="module")
def ext():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from pdattention_b200.ops import _ext

    return _ext.require()


def philox_words(seed: int, offset: int, blocks: np.ndarray) -> np.ndarray:
    """[n, 4] Philox4x32-10 words of counter blocks (block, offset) under key seed."""
    b = blocks.astype(np.uint64)
    c = [b & M32, b >> np.uint64(32), np.full_like(b, offset & 0xFFFFFFFF), np.full_like(b, offset >> 32)]
    k0, k1 = np.uint64(seed & 0xFFFFFFFF), np.uint64(seed >> 32)
    for _ in range(10):
        p0 = c[0] * np.uint64(0xD2511F53)
        p1 = c[2] * np.uint64(0xCD9E8D57)
        c = [(p1 >> np.uint64(32)) ^ c[1] ^ k0, p1 & M32, (p0 >> np.uint64(32)) ^ c[3] ^ k1, p0 & M32]
        k0 = (k0 + np.uint64(0x9E3779B9)) & M32
        k1 = (k1 + np.uint64(0xBB67AE85)) & M32
    return np.stack(c, axis=1)


def keep_mask(seed: int, offset: int, n: int, p: float) -> np.ndarray:
    e = np.arange(n, dtype=np.uint64)
    words = philox_words(seed, offset, e >> np.uint64(2))[np.arange(n), (e & np.uint64(3)).astype(np.int64)]
    return (words >> np.uint64(8)) >= np.uint64(round(p * (1 << 24)))


def test_dropout_mask_is_the_philox_stream(ext):
    n, p, seed, offset = 10_007, 0.3, 123456789012345, 77
    x = torch.ones(n, device="cuda", dtype=torch.bfloat16)
    y = torch.empty_like(x)
    ext.dropout(x, y, p, seed, offset)
    want = keep_mask(seed, offset, n, p)
    got = (y.float() != 0).cpu().numpy()
    assert (got == want).all()
    assert abs(got.mean() - (1 - p)) < 0.02
    kept = y.float()[torch.from_numpy(want).cuda()]
    assert torch.allclose(kept, torch.full_like(kept, 1 / (1 - p)), rtol=1e-2)


def test_dropout_add_matches_the_mask(ext):
    n, p, seed, offset = 4099, 0.1, 5, 9
    res = torch.randn(n, device="cuda").bfloat16()
    x = torch.randn(n, device="cuda").bfloat16()
    y = torch.empty_like(x)
    ext.dropout_add(res, x, y, p, seed, offset)
    mask = torch.from_numpy(keep_mask(seed, offset, n, p)).cuda()
    ref = res.float() + torch.where(mask, x.float() / (1 - p), torch.zeros_like(x.float()))
    assert torch.allclose(y.float(), ref, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("head_dim,T,padded", [(64, 150, False), (32, 97, True)])
def test_attention_dropout_forward_and_backward(ext, head_dim, T, padded):
    torch.manual_seed(7)
    B, H, p, seed, offset = 2, 3, 0.2, 42, 3
    d = H * head_dim
    qkv = (torch.randn(B, T, 3 * d, device="cuda") * 0.5).bfloat16()
    valid = torch.ones(B, T, device="cuda", dtype=torch.uint8)
    if padded:
        valid[1, T - 20:] = 0
    kv = valid if padded else None
    q, k, v = qkv[..., :d], qkv[..., d:2 * d], qkv[..., 2 * d:]
    scale = 1 / math.sqrt(head_dim)
    out, lse = ext.attention_fwd(q, k, v, H, H, head_dim, None, None, None, None, kv, scale, p, seed, offset)
    mask = torch.from_numpy(keep_mask(seed, offset, B * H * T * T, p)).cuda().view(B, H, T, T)

    qf, kf, vf = (t.float().view(B, T, H, head_dim).transpose(1, 2).requires_grad_(True) for t in (q, k, v))
    s = qf @ kf.transpose(-1, -2) * scale
    hide = torch.ones(T, T, device="cuda", dtype=torch.bool).triu(1)[None, None]
    hide = hide | (valid == 0)[:, None, None, :]
    probs = torch.softmax(s.masked_fill(hide, float("-inf")), dim=-1)
    ref = (probs * mask / (1 - p)) @ vf
    ref_out = ref.transpose(1, 2).reshape(B, T, d)
    assert torch.allclose(out.float(), ref_out, atol=2e-2, rtol=2e-2), (out.float() - ref_out).abs().max()

    dout = torch.randn(B, T, d, device="cuda").bfloat16()
    (dqkv,) = ext.attention_bwd(dout, q, k, v, out, lse, H, head_dim, None, None, None, None, kv, scale, p, seed,
                                offset)
    ref_out.backward(dout.float())
    for i, t in enumerate((qf, kf, vf)):
        want = t.grad.transpose(1, 2).reshape(B, T, d)
        got = dqkv[..., i * d:(i + 1) * d].float()
        tol = 3e-2 * want.abs().max().item() + 1e-3
        assert (got - want).abs().max().item() <= tol, ("qkv"[i], (got - want).abs().max().item(), tol)


def _variant(vocab: int, kind: str):
    cfg = copy.deepcopy(tiny_config(vocab))
    cfg.n_layers = 3
    cfg.dropout = 0.1
    if kind == "tdx":
        cfg.model_variant, cfg.n_vanilla_layers, cfg.n_mixed_layers = "tdx_pra", 1, 0
    else:
        cfg.model_variant, cfg.n_vanilla_layers, cfg.n_mixed_layers = "custom", 1, 1
        cfg.pra_layer_ids = (1, 2)
    cfg.__post_init__()
    return cfg


@pytest.mark.parametrize("kind", ["tdx", "mixed"])
def test_vanilla_and_mixed_blocks_match_object_path(ext, tmp_path, kind):
    torch.manual_seed(12)
    tok, batch = tiny_batch(Path(tmp_path))
    cfg = _variant(tok.vocab_size, kind)
    reference = TinyPRAModel(copy.deepcopy(cfg)).cuda().eval()
    device_model = TinyPRAModel(copy.deepcopy(cfg)).cuda().eval()
    device_model.load_state_dict(reference.state_dict())
    attach_device_runtime(device_model)
    rt = device_model._device_runtime
    assert rt is not None and not rt.uniform_pra
    assert rt.kinds == (["vanilla", "pra", "pra"] if kind == "tdx" else ["vanilla", "mixed", "pra"])
    with torch.no_grad():
        ref_loss, ref_out = _pra_batch_step(reference, batch, "cuda", tok, ResolverServiceConfig(), None)
        dev_loss, dev_out = _pra_batch_step(device_model, batch, "cuda", tok, ResolverServiceConfig(), None)
    b, t = batch["input_ids"].shape
    dev_logits = rt.logits(dev_out["hidden"], b, t).float()
    ref_logits = ref_out["logits"].float()
    valid = batch["attention_mask"].bool().cuda()
    err = (dev_logits - ref_logits).abs()[valid]
    assert err.max() <= 0.05 * ref_logits.abs()[valid].max(), err.max()
    assert abs(dev_loss.item() - ref_loss.item()) < 0.03 * abs(ref_loss.item())


def test_dropout_training_on_the_device_path(ext, tmp_path):
    torch.manual_seed(13)
    tok, batch = tiny_batch(Path(tmp_path))
    model = TinyPRAModel(_variant(tok.vocab_size, "mixed")).cuda()
    attach_device_runtime(model)
    model.train()
    opt = model.build_optimizer(TrainConfig(device="cuda", learning_rate=3e-3))
    rt = model._device_runtime
    losses = []
    for _ in range(12):
        opt.zero_grad()
        loss, _ = _pra_batch_step(model, batch, "cuda", tok, ResolverServiceConfig(), None)
        loss.backward()
        assert torch.isfinite(rt.flat.grad.float()).all()
        opt.step()
        losses.append(loss.item())
    assert rt.dropout_streams.offset > 0  # dropout streams were drawn
    assert losses[-1] < 0.8 * losses[0], losses


def test_cross_attention_transport_matches_object_path(ext, tmp_path):
    """Legacy transport: separately normalised memory attention through mem_o_proj, scaled by
    memory_alpha, next to the local attention (the ragged kernel with every local key masked)."""
    torch.manual_seed(14)
    tok, batch = tiny_batch(Path(tmp_path))
    cfg = copy.deepcopy(tiny_config(tok.vocab_size))
    cfg.memory_transport, cfg.memory_alpha = "cross_attention", 0.5
    cfg.__post_init__()
    reference = TinyPRAModel(copy.deepcopy(cfg)).cuda().eval()
    device_model = TinyPRAModel(copy.deepcopy(cfg)).cuda().eval()
    device_model.load_state_dict(reference.state_dict())
    attach_device_runtime(device_model)
    rt = device_model._device_runtime
    assert rt is not None and rt.cross_attention and "mem_o" in rt.layers[0]
    with torch.no_grad():
        ref_loss, ref_out = _pra_batch_step(reference, batch, "cuda", tok, ResolverServiceConfig(), None)
        dev_loss, dev_out = _pra_batch_step(device_model, batch, "cuda", tok, ResolverServiceConfig(), None)
    assert int(rt.last_routing[0].ints[0].sum()) > 0  # memory was materialised
    b, t = batch["input_ids"].shape
    dev_logits = rt.logits(dev_out["hidden"], b, t).float()
    ref_logits = ref_out["logits"].float()
    valid = batch["attention_mask"].bool().cuda()
    err = (dev_logits - ref_logits).abs()[valid]
    assert err.max() <= 0.05 * ref_logits.abs()[valid].max(), err.max()
    # and it trains (gradients flow through both branches)
    device_model.train()
    opt = device_model.build_optimizer(TrainConfig(device="cuda", learning_rate=1e-3))
    opt.zero_grad()
    loss, _ = _pra_batch_step(device_model, batch, "cuda", tok, ResolverServiceConfig(), None)
    loss.backward()
    gw = rt.layers[0]["mem_o"].gw
    assert torch.isfinite(rt.flat.grad.float()).all() and float(gw.float().abs().sum()) > 0


@pytest.mark.parametrize("profile", ["tiny", "medium", "td_sa_tiny", "tdx_pra_tiny", "td_pra_tiny", "kvqa_tiny"])
def test_named_profiles_match_object_path(ext, tmp_path, profile):
    """The config.yml model profiles (head widths 16 / 32 / 64, vanilla and mixed blocks) on the
    device path against the fp32 object path in eval mode."""
    from pdattention_b200.cli import build_pra_config, load_config
    from pdattention_b200.data import PRADataModule, WordIdTokenizer
    from pdattention_b200.data.generators import generate_hierarchical_tokens

    root = Path(tmp_path)
    generate_hierarchical_tokens(root / "synthetic_hierarchical_tokens", examples=4, doc_tokens=24, prompt_tokens=40,
                                 vocab=300, roots=2, children=1, grandchildren=1)
    tok = WordIdTokenizer(300)
    dm = PRADataModule("synthetic_hierarchical_tokens", str(root), batch_size=4, max_seq_len=64, tokenizer=tok,
                       shuffle=False).load()
    batch = next(iter(dm._loader(dm.dataset, shuffle=False)))
    path = Path(__file__).resolve().parents[1] / "config" / "config.yml"
    cfg = build_pra_config(load_config(str(path), profile), vocab_size=tok.vocab_size, batch_size=4, lr=1e-3,
                           steps=1, device="cuda")
    torch.manual_seed(31)
    reference = TinyPRAModel(copy.deepcopy(cfg)).cuda().eval()
    device_model = TinyPRAModel(copy.deepcopy(cfg)).cuda().eval()
    device_model.load_state_dict(reference.state_dict())
    attach_device_runtime(device_model)
    rt = device_model._device_runtime
    assert rt is not None, profile
    with torch.no_grad():
        _, ref_out = _pra_batch_step(reference, batch, "cuda", tok, ResolverServiceConfig(), None)
        _, dev_out = _pra_batch_step(device_model, batch, "cuda", tok, ResolverServiceConfig(), None)
    b, t = batch["input_ids"].shape
    dev_logits = rt.logits(dev_out["hidden"], b, t).float()
    ref_logits = ref_out["logits"].float()
    valid = batch["attention_mask"].bool().cuda()
    err = (dev_logits - ref_logits).abs()[valid]
    assert err.max() <= 0.05 * ref_logits.abs()[valid].max(), (profile, err.max())
