"""PRA-Llama family oracle: architecture parity with Hugging Face and memory semantics (CPU)."""

import pytest
import torch

from pdattention_b200.models.llama import (PRALlamaConfig, PRALlamaReference, hf_config, select_chunks, tiny_llama)


def _hf_model(cfg):
    import transformers

    hcfg = hf_config(cfg)
    cls = {"llama": transformers.LlamaForCausalLM, "mistral": transformers.MistralForCausalLM,
           "qwen2": transformers.Qwen2ForCausalLM}[cfg.family]
    hcfg._attn_implementation = "eager"
    return cls(hcfg).eval()


@pytest.mark.parametrize("family", ["llama", "mistral", "qwen2"])
def test_no_memory_forward_matches_hugging_face(family):
    cfg = tiny_llama(family=family, attention_bias=(family == "qwen2"))
    ours = PRALlamaReference(cfg).eval()
    ours.reset_parameters(seed=0)
    hf = _hf_model(cfg)
    missing, unexpected = hf.load_state_dict(ours.state_dict(), strict=False)
    assert not unexpected and all("rotary" in m for m in missing), (missing, unexpected)
    ids = torch.randint(0, cfg.vocab_size, (2, 24), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = hf(ids).logits
    got = ours(ids)
    assert torch.allclose(got, ref, atol=1e-4, rtol=1e-4), (got - ref).abs().max()


def test_padding_mask_matches_unpadded_rows():
    cfg = tiny_llama()
    model = PRALlamaReference(cfg).eval()
    ids = torch.randint(0, cfg.vocab_size, (1, 10))
    padded = torch.cat([ids, torch.zeros(1, 6, dtype=torch.long)], dim=1)
    mask = torch.cat([torch.ones(1, 10), torch.zeros(1, 6)], dim=1).long()
    full = model(ids)
    part = model(padded, attention_mask=mask)
    assert torch.allclose(full, part[:, :10], atol=1e-5)


def test_routing_picks_highest_cosine_then_chunk_order():
    cfg = tiny_llama(top_k_chunks=2)
    gist = torch.tensor([[1.0, 0.0], [0.0, 1.0], [0.7, 0.7], [1.0, 0.0]])
    query = torch.tensor([[1.0, 0.05]])
    picked = select_chunks(cfg, query, gist, [[0, 1, 2, 3]])
    assert picked == [[0, 3]]  # chunks 0 and 3 tie on score; both beat chunk 2; returned in chunk order
    picked = select_chunks(cfg, query, gist, [[1, 2]])
    assert picked == [[1, 2]]
    cfg_budget = tiny_llama(top_k_chunks=3, memory_budget_tokens=cfg.chunk_tokens)
    assert select_chunks(cfg_budget, query, gist, [[0, 1, 2, 3]]) == [[0]]


def test_memory_changes_output_only_through_selected_chunks():
    torch.manual_seed(0)
    cfg = tiny_llama(top_k_chunks=2)
    model = PRALlamaReference(cfg).eval()
    chunks = torch.randint(0, cfg.vocab_size, (5, cfg.chunk_tokens))
    lengths = torch.tensor([16, 16, 9, 16, 12])
    mem = model.encode_chunks(chunks, lengths)
    assert mem.gist[0].shape == (5, cfg.kv_dim)
    mem.namespace = [[0, 1, 2, 3, 4], [2, 4]]
    ids = torch.randint(0, cfg.vocab_size, (2, 12))
    logits, sel = model(ids, memory=mem, return_selection=True)
    assert len(sel) == cfg.num_hidden_layers and all(len(s[1]) <= 2 for s in sel)
    # rows' outputs depend on memory: removing the namespace changes them
    mem_empty = model.encode_chunks(chunks, lengths)
    mem_empty.namespace = [[], []]
    plain = model(ids, memory=mem_empty)
    assert not torch.allclose(logits, plain)
    assert torch.allclose(plain, model(ids), atol=1e-6)


def test_config_presets_and_parameter_counts():
    from pdattention_b200.models.llama import llama3_8b, mistral_7b, qwen2_7b

    assert abs(llama3_8b().parameter_count() / 1e9 - 8.03) < 0.05
    assert abs(mistral_7b().parameter_count() / 1e9 - 7.25) < 0.05
    assert abs(qwen2_7b().parameter_count() / 1e9 - 7.62) < 0.05
    with pytest.raises(ValueError):
        PRALlamaConfig(num_attention_heads=6, num_key_value_heads=4)


def test_incremental_reference_matches_full_forward_without_memory():
    from pdattention_b200.models.llama import reference_step

    cfg = tiny_llama()
    model = PRALlamaReference(cfg).eval()
    ids = torch.randint(0, cfg.vocab_size, (9,))
    full = model(ids[None])[0]
    cache = [[None, None] for _ in range(cfg.num_hidden_layers)]
    a, _ = reference_step(model, ids[:6], cache, None, None)
    b, _ = reference_step(model, ids[6:], cache, None, None)
    assert torch.allclose(torch.cat([a, b]), full, atol=1e-5)


def test_long_prompt_plan_splits_head_and_tail():
    from pdattention_b200.inference.long_prompt import plan_long_prompts

    prompts = [list(range(1, 51)), list(range(100, 110))]
    plan = plan_long_prompts(prompts, direct_window=12, chunk_tokens=16, max_positions=40)
    assert plan.chunks.shape == (3, 16)  # row 0: 38 head tokens -> 16 + 16 + 6
    assert plan.chunk_lengths.tolist() == [16, 16, 6]
    assert plan.ns_start.tolist() == [0, 3] and plan.ns_end.tolist() == [3, 3]
    assert plan.tails[0].tolist() == list(range(39, 51)) and plan.tail_lengths.tolist() == [12, 10]
    assert plan.position_offset.tolist() == [0, 0]  # 50 > 40 native positions: the tail restarts at 0
    plan = plan_long_prompts(prompts, direct_window=12, chunk_tokens=16, max_positions=64)
    assert plan.position_offset.tolist() == [38, 0]
    assert plan.chunk_ids[0] == "pra://implicit/prompt/head#chunk=0"
