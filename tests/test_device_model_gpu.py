"""TinyGPT-PRA device path against the fp32 object path (same weights) on a GPU."""

import copy
from pathlib import Path

import pytest
import torch

from pdattention_b200.config import ResolverServiceConfig, TrainConfig
from pdattention_b200.models import TinyPRAModel
from pdattention_b200.models.fastpath import attach_device_runtime
from pdattention_b200.pra_train import _pra_batch_step
from pdattention_b200.smoke import tiny_batch, tiny_config, tiny_training_step

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch.device("cuda", 0)


def test_smoke_step(cuda):
    assert torch.isfinite(torch.tensor(tiny_training_step(cuda)))


def test_device_loss_matches_object_path(cuda, tmp_path):
    torch.manual_seed(1)
    tok, batch = tiny_batch(Path(tmp_path))
    cfg = tiny_config(tok.vocab_size)
    reference = TinyPRAModel(copy.deepcopy(cfg)).to(cuda).eval()
    device_model = TinyPRAModel(copy.deepcopy(cfg)).to(cuda)
    device_model.load_state_dict(reference.state_dict())
    attach_device_runtime(device_model)
    assert device_model._device_runtime is not None
    with torch.no_grad():
        ref_loss, _ = _pra_batch_step(reference, batch, "cuda", tok, ResolverServiceConfig(), None)
        dev_loss, out = _pra_batch_step(device_model, batch, "cuda", tok, ResolverServiceConfig(), None)
    assert abs(dev_loss.item() - ref_loss.item()) < 0.03 * abs(ref_loss.item()), (dev_loss.item(), ref_loss.item())
    # the device routing saw every row's namespace and materialised memory
    rt = device_model._device_runtime
    lens = rt.last_routing[0].ints[0]
    assert int(lens.sum()) > 0


def test_device_training_reduces_loss(cuda, tmp_path):
    torch.manual_seed(2)
    tok, batch = tiny_batch(Path(tmp_path))
    model = TinyPRAModel(tiny_config(tok.vocab_size)).to(cuda)
    attach_device_runtime(model)
    opt = model.build_optimizer(TrainConfig(device="cuda", learning_rate=3e-3))
    losses = []
    for _ in range(15):
        opt.zero_grad()
        loss, _ = _pra_batch_step(model, batch, "cuda", tok, ResolverServiceConfig(), None)
        loss.backward()
        opt.step()
        losses.append(loss.item())
    assert losses[-1] < 0.7 * losses[0], losses


def test_checkpoint_roundtrip_keeps_reference_layout(cuda, tmp_path):
    tok, _ = tiny_batch(Path(tmp_path))
    model = TinyPRAModel(tiny_config(tok.vocab_size)).to(cuda)
    attach_device_runtime(model)
    keys = set(TinyPRAModel(tiny_config(tok.vocab_size)).state_dict())
    assert set(model.state_dict()) == keys
    state = {k: v.clone() for k, v in model.state_dict().items()}
    other = TinyPRAModel(tiny_config(tok.vocab_size)).to(cuda)
    attach_device_runtime(other)
    other.load_state_dict(state)
    assert torch.equal(other._device_runtime.flat.shadow, model._device_runtime.flat.shadow)


def test_native_stack_executor_matches_autograd_path(cuda, tmp_path):
    """The C++ block-stack executor (no-grad forwards, cache build) equals the autograd path."""
    torch.manual_seed(3)
    tok, batch = tiny_batch(Path(tmp_path))
    model = TinyPRAModel(tiny_config(tok.vocab_size)).to(cuda)
    attach_device_runtime(model)
    rt = model._device_runtime
    memory, _, _ = rt.build_memory(batch["metadata"], tok, ResolverServiceConfig())
    ids = batch["input_ids"].to(cuda)
    mask = batch["attention_mask"].to(cuda)
    with torch.enable_grad():
        ref = rt.prompt_forward(ids, mask, memory).float()
        ref_routing = {k: v.mem_idx.clone() for k, v in rt.last_routing.items()}
        ref_lens = {k: v.ints[0].clone() for k, v in rt.last_routing.items()}
    with torch.no_grad():
        got = rt.prompt_forward(ids, mask, memory).float()
    assert set(rt.last_routing) == set(ref_routing)
    for li, routing in rt.last_routing.items():
        assert torch.equal(routing.ints[0], ref_lens[li])
        for row in range(ids.shape[0]):
            n = int(ref_lens[li][row])
            assert torch.equal(routing.mem_idx[row, :n], ref_routing[li][row, :n])
    assert torch.allclose(got, ref, atol=2e-2, rtol=2e-2), (got - ref).abs().max()


def test_native_train_stack_matches_per_layer_autograd(cuda, tmp_path):
    """One autograd node over the native block stack gives the per-layer autograd path's loss and
    (up to the rounding of the fused residual-gradient add) its gradients."""
    from pdattention_b200.models import fastpath

    torch.manual_seed(4)
    tok, batch = tiny_batch(Path(tmp_path))
    model = TinyPRAModel(tiny_config(tok.vocab_size)).to(cuda)
    attach_device_runtime(model)
    opt = model.build_optimizer(TrainConfig(device="cuda", learning_rate=1e-3))
    rt = model._device_runtime
    results = {}
    try:
        for native in (True, False):
            fastpath._NATIVE_TRAIN_STACK = native
            opt.zero_grad()
            loss, _ = _pra_batch_step(model, batch, "cuda", tok, ResolverServiceConfig(), None)
            loss.backward()
            lens = rt.last_routing[0].ints[0].clone()
            results[native] = (loss.detach().clone(), rt.flat.grad.float().clone(), lens)
    finally:
        fastpath._NATIVE_TRAIN_STACK = True
    assert torch.equal(results[True][0], results[False][0])
    assert torch.equal(results[True][2], results[False][2]) and int(results[True][2].sum()) > 0
    g_native, g_python = results[True][1], results[False][1]
    assert torch.isfinite(g_native).all()
    err = (g_native - g_python).abs().max().item()
    assert err <= 2e-2 * g_python.abs().max().item(), err


def test_layer_synchronous_cache_build_matches_wave_build(cuda, tmp_path, monkeypatch):
    """One pass over every chunk, layer by layer, gives the memory an entry-by-entry (wave) build gives."""
    from pdattention_b200.models import fastpath

    torch.manual_seed(5)
    tok, batch = tiny_batch(Path(tmp_path))
    model = TinyPRAModel(tiny_config(tok.vocab_size)).to(cuda)
    attach_device_runtime(model)
    rt = model._device_runtime
    built = {}
    for sync in (False, True):
        monkeypatch.setattr(fastpath, "_LAYER_SYNC", sync)
        with torch.no_grad():
            memory, _, _ = rt.build_memory(batch["metadata"], tok, ResolverServiceConfig())
        torch.cuda.synchronize()
        built[sync] = (memory.pool.float().clone(), memory.gists_all.clone(), memory.gist_count_all.clone())
    assert len(rt.plan_batch(batch["metadata"], tok).waves) == 1  # one encode group in layer-synchronous mode
    (pool_a, gists_a, count_a), (pool_b, gists_b, count_b) = built[False], built[True]
    assert torch.equal(count_a, count_b)
    assert torch.allclose(pool_a, pool_b, atol=2e-2, rtol=2e-2), (pool_a - pool_b).abs().max()
    assert torch.allclose(gists_a, gists_b, atol=2e-2, rtol=2e-2), (gists_a - gists_b).abs().max()


def test_device_logits_and_selected_chunks_match_object_path(cuda, tmp_path):
    """Model level: bf16 device logits against the fp32 object path (which equals the reference
    oracle on CPU), and the chunk ids each layer selects for each row."""
    torch.manual_seed(11)
    tok, batch = tiny_batch(Path(tmp_path))
    cfg = tiny_config(tok.vocab_size)
    reference = TinyPRAModel(copy.deepcopy(cfg)).to(cuda).eval()
    device_model = TinyPRAModel(copy.deepcopy(cfg)).to(cuda)
    device_model.load_state_dict(reference.state_dict())
    attach_device_runtime(device_model)
    with torch.no_grad():
        _, ref_out = _pra_batch_step(reference, batch, "cuda", tok, ResolverServiceConfig(), None)
        _, dev_out = _pra_batch_step(device_model, batch, "cuda", tok, ResolverServiceConfig(), None)
    rt = device_model._device_runtime
    b, t = batch["input_ids"].shape
    dev_logits = rt.logits(dev_out["hidden"], b, t).float()
    ref_logits = ref_out["logits"].float()
    valid = batch["attention_mask"].bool().to(cuda)
    err = (dev_logits - ref_logits).abs()[valid]
    assert err.max() <= 0.05 * ref_logits.abs()[valid].max(), err.max()
    expected = reference.selected_chunks_by_layer()
    memory = dev_out["memory"]
    for layer, rows in expected.items():
        routing = rt.last_routing[layer]
        same = 0
        for row in range(b):
            count = int(routing.ints[1, row])
            got = sorted(memory.chunks[int(c)].chunk_id for c in routing.sel_i[0, row, :count].tolist())
            want = sorted(hit.chunk_id for hit in rows[row])
            same += got == want
        # layer 0 routes queries that differ from the fp32 ones only by bf16 rounding
        assert same == b if layer == 0 else same >= 0.75 * b, (layer, same, b)


def test_cpu_resident_kv_tier_matches_gpu_residency(cuda, tmp_path):
    """kv_cache_residency="cpu": the encoded pool lives in pinned host memory and the attention
    kernels gather the selected rows over the host link; the loss and its gradients equal the
    device-resident run, and no cached K/V stays on the device."""
    torch.manual_seed(21)
    tok, batch = tiny_batch(Path(tmp_path))
    results = {}
    for residency in ("gpu", "cpu"):
        cfg = tiny_config(tok.vocab_size)
        cfg.kv_cache_residency = residency
        torch.manual_seed(22)
        model = TinyPRAModel(cfg).to(cuda)
        attach_device_runtime(model)
        assert model._device_runtime is not None
        opt = model.build_optimizer(TrainConfig(device="cuda", learning_rate=1e-3))
        opt.zero_grad()
        loss, out = _pra_batch_step(model, batch, "cuda", tok, ResolverServiceConfig(), None)
        loss.backward()
        torch.cuda.synchronize()
        mem = out["memory"]
        results[residency] = (loss.item(), model._device_runtime.flat.grad.float().clone(), out["metrics"],
                              mem.pool.is_cuda)
    (l_gpu, g_gpu, m_gpu, on_gpu), (l_cpu, g_cpu, m_cpu, on_cpu_dev) = results["gpu"], results["cpu"]
    assert on_gpu and not on_cpu_dev
    assert l_cpu == l_gpu
    assert torch.equal(g_cpu, g_gpu)
    assert m_cpu["gpu_cached_kv_bytes"] == 0 and m_cpu["cached_kv_bytes"] == m_gpu["cached_kv_bytes"] > 0


@pytest.mark.parametrize("mode", ["last", "ref_end"])
def test_single_token_gists_match_object_path(cuda, tmp_path, mode):
    """``last`` / ``ref_end`` gists: a chunk's gist is one token's key (the last one, or the single
    reference terminator); device logits and per-layer selections against the object path."""
    import json

    from pdattention_b200.data import PRADataModule, WordIdTokenizer
    from pdattention_b200.data.generators import generate_hierarchical_tokens

    root = Path(tmp_path)
    stage = generate_hierarchical_tokens(root / "synthetic_hierarchical_tokens", examples=4, doc_tokens=40,
                                         prompt_tokens=95, vocab=500, roots=2, children=1, grandchildren=2)
    docs = [json.loads(line) for line in (stage / "documents.jsonl").read_text().splitlines() if line.strip()]
    with (stage / "documents.jsonl").open("w") as fh:
        for doc in docs:  # the terminator mid-document, so "ref_end" and "last" pick different tokens
            words = doc["text"].split()
            doc["text"] = " ".join(words[:7] + ["<REF_END>"] + words[7:])
            fh.write(json.dumps(doc) + "\n")
    tok = WordIdTokenizer(500)
    dm = PRADataModule("synthetic_hierarchical_tokens", str(root), batch_size=4, max_seq_len=256, tokenizer=tok,
                       shuffle=False).load()
    batch = next(iter(dm._loader(dm.dataset, shuffle=False)))
    cfg = tiny_config(tok.vocab_size)
    cfg.gist_mode, cfg.gists_per_chunk, cfg.chunking_mode = mode, 1, "none"
    torch.manual_seed(23)
    reference = TinyPRAModel(copy.deepcopy(cfg)).to(cuda).eval()
    device_model = TinyPRAModel(copy.deepcopy(cfg)).to(cuda)
    device_model.load_state_dict(reference.state_dict())
    attach_device_runtime(device_model)
    rt = device_model._device_runtime
    assert rt is not None
    with torch.no_grad():
        _, ref_out = _pra_batch_step(reference, batch, "cuda", tok, ResolverServiceConfig(), None)
        _, dev_out = _pra_batch_step(device_model, batch, "cuda", tok, ResolverServiceConfig(), None)
    b, t = batch["input_ids"].shape
    dev_logits = rt.logits(dev_out["hidden"], b, t).float()
    ref_logits = ref_out["logits"].float()
    valid = batch["attention_mask"].bool().to(cuda)
    err = (dev_logits - ref_logits).abs()[valid]
    assert err.max() <= 0.05 * ref_logits.abs()[valid].max(), err.max()
    memory = dev_out["memory"]
    expected = reference.selected_chunks_by_layer()
    routing = rt.last_routing[0]
    for row in range(b):
        count = int(routing.ints[1, row])
        got = sorted(memory.chunks[int(c)].chunk_id for c in routing.sel_i[0, row, :count].tolist())
        assert got == sorted(hit.chunk_id for hit in expected[0][row])


def test_global_chunk_search_matches_object_path(cuda, tmp_path):
    """search_strategy="global_chunks": one ranking of every chunk under the distinct-URI and
    per-URI limits (route kernel) against the object path's selections and logits."""
    torch.manual_seed(24)
    tok, batch = tiny_batch(Path(tmp_path))
    cfg = tiny_config(tok.vocab_size)
    cfg.search_strategy, cfg.top_k_references, cfg.top_k_chunks_per_reference = "global_chunks", 2, 2
    reference = TinyPRAModel(copy.deepcopy(cfg)).to(cuda).eval()
    device_model = TinyPRAModel(copy.deepcopy(cfg)).to(cuda)
    device_model.load_state_dict(reference.state_dict())
    attach_device_runtime(device_model)
    rt = device_model._device_runtime
    assert rt is not None
    with torch.no_grad():
        _, ref_out = _pra_batch_step(reference, batch, "cuda", tok, ResolverServiceConfig(), None)
        _, dev_out = _pra_batch_step(device_model, batch, "cuda", tok, ResolverServiceConfig(), None)
    b, t = batch["input_ids"].shape
    dev_logits = rt.logits(dev_out["hidden"], b, t).float()
    ref_logits = ref_out["logits"].float()
    valid = batch["attention_mask"].bool().to(cuda)
    err = (dev_logits - ref_logits).abs()[valid]
    assert err.max() <= 0.05 * ref_logits.abs()[valid].max(), err.max()
    memory = dev_out["memory"]
    expected = reference.selected_chunks_by_layer()
    routing = rt.last_routing[0]
    for row in range(b):
        count = int(routing.ints[1, row])
        got = [memory.chunks[int(c)].chunk_id for c in routing.sel_i[0, row, :count].tolist()]
        want = [hit.chunk_id for hit in expected[0][row]]
        assert sorted(got) == sorted(want), (row, got, want)
        assert len({c.split("#")[0] for c in got}) <= 2
