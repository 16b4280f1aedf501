"""The Llama engine's one-time weight preparation, on CPU.

An engine appends the routing-query rows to each layer's QKV weight, interleaves the gate / up
rows in runs of 64 (so a decode-GEMM tile holds matching gate and up features) and multiplies
the RMSNorm weights into the projections after them.  These tests check that the prepared
weights still compute the same functions as the originals (fp32 reference), and that a second
engine over the same weight set prepares nothing twice.
"""

import torch

from pdattention_b200.inference.llama_engine import LlamaWeights, PRALlamaEngine
from pdattention_b200.models.llama import PRALlamaReference, tiny_llama


def _model():
    cfg = tiny_llama(head_dim=64, hidden_size=128, num_attention_heads=4, num_key_value_heads=2, chunk_tokens=16,
                     top_k_chunks=3)
    model = PRALlamaReference(cfg).eval()
    model.reset_parameters(seed=3, std=0.08)
    with torch.no_grad():  # non-trivial norm weights, so folding them matters
        for layer in model.model.layers:
            layer.input_layernorm.weight.uniform_(0.5, 1.5)
            layer.post_attention_layernorm.weight.uniform_(0.5, 1.5)
    return cfg, model


def _rms(x, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)


def test_prepared_weights_compute_the_original_projections():
    cfg, model = _model()
    weights = LlamaWeights.from_reference(model, "cpu")
    engine = PRALlamaEngine(weights, "cpu")
    assert weights.norm_folded and weights.mlp_block == 64
    x = torch.randn(5, cfg.hidden_size)
    h = _rms(x, cfg.rms_norm_eps)
    f = cfg.intermediate_size
    for layer, lw in zip(model.model.layers, weights.layers):
        a, m = layer.self_attn, layer.mlp
        # QKV (+ routing rows) on the unit-weight norm equals the original projections of the weighted norm
        got = h @ lw.qkv_route.float().t()
        hw = h * layer.input_layernorm.weight
        qd, kd = engine.q_dim, engine.kv_dim
        want_qkv = torch.cat([hw @ a.q_proj.weight.t(), hw @ a.k_proj.weight.t(), hw @ a.v_proj.weight.t()], -1)
        tol = 3e-2 * want_qkv.abs().max().item()
        assert (got[:, : qd + 2 * kd] - want_qkv).abs().max() < tol
        # routing rows: the KV-group mean of the query rows
        q = want_qkv[:, :qd].view(5, cfg.num_key_value_heads, cfg.group, cfg.head_dim).mean(2).reshape(5, -1)
        assert (got[:, qd + 2 * kd:] - q).abs().max() < tol
        # gate / up in runs of 64, with the post-attention norm weight folded in
        gu = (h @ lw.gate_up.float().t()).view(5, f // 64, 2, 64)
        hp = h * layer.post_attention_layernorm.weight
        gate, up = hp @ m.gate_proj.weight.t(), hp @ m.up_proj.weight.t()
        tol = 3e-2 * max(gate.abs().max().item(), up.abs().max().item())
        assert (gu[:, :, 0].reshape(5, f) - gate).abs().max() < tol
        assert (gu[:, :, 1].reshape(5, f) - up).abs().max() < tol


def test_a_second_engine_prepares_nothing_twice():
    cfg, model = _model()
    weights = LlamaWeights.from_reference(model, "cpu")
    PRALlamaEngine(weights, "cpu")
    snapshot = [(lw.qkv_route.clone(), lw.gate_up.clone()) for lw in weights.layers]
    PRALlamaEngine(weights, "cpu")
    for (qkv, gu), lw in zip(snapshot, weights.layers):
        assert torch.equal(qkv, lw.qkv_route)
        assert torch.equal(gu, lw.gate_up)
        assert lw.qkv.data_ptr() == lw.qkv_route.data_ptr()  # q|k|v stays a view of the fused weight
