"""Pins the MoE oracle (oracle/moe.py) to Hugging Face transformers' own
sparse-MoE blocks run in BF16 on the CPU -- the ground truth the reference
validates its router and expert math against (tests/test_f33_router_oracle.py
:30-40 of the reference) -- for the three families the reference runs:

  generic  OlmoeSparseMoeBlock           (runtime/layer_runner.py run_moe_mlp)
  qwen35   Qwen3_5MoeSparseMoeBlock      (runtime/qwen35.py _route_experts/_moe)
  glm      GlmMoeDsaMoE                  (runtime/glm.py _route_experts/_glm_mlp_residual)

Same weights and inputs on both sides.  The routes must be the same expert
sets; with HF's rounding points (`hf_rounding=True`: SiLU rounded once, fp32
route weights, ascending expert order) the oracle must reproduce HF bit for
bit (exactly for one token; with many tokens per expert, CPU BF16 GEMMs sum
in a different fp32 order than a plain matmul, which flips a few outputs by
one BF16 ulp, so the bound there is rel-L2 1e-3), and with the reference's
rounding points it must stay within rel-L2 1e-2 of HF (the BASELINE
tolerance) -- the remaining gap is BF16 rounding only.
"""

from __future__ import annotations

import pytest
import torch

from oracle import moe as om

transformers = pytest.importorskip("transformers")
bf16 = torch.bfloat16
TOL = 1e-2


def _experts(E, H, I, std, seed):
    g = torch.Generator().manual_seed(seed)
    return [tuple((torch.randn(s, generator=g) * std).to(bf16) for s in ((I, H), (I, H), (H, I))) for _ in range(E)]


def _load_experts(mod, ex):
    with torch.no_grad():
        for e, (wg, wu, wd) in enumerate(ex):
            mod.gate_up_proj[e].copy_(torch.cat([wg, wu], 0))
            mod.down_proj[e].copy_(wd)


def _mlp(mod, trip):
    with torch.no_grad():
        mod.gate_proj.weight.copy_(trip[0])
        mod.up_proj.weight.copy_(trip[1])
        mod.down_proj.weight.copy_(trip[2])


def _same_routes(a, b):
    return [sorted(r) for r in a.tolist()] == [sorted(r) for r in b.tolist()]


def _pinned(hf_mode: torch.Tensor, hf: torch.Tensor, T: int) -> bool:
    return torch.equal(hf_mode, hf) if T == 1 else om.rel_l2(hf_mode, hf) < 1e-3


@pytest.mark.parametrize("T,norm", [(1, True), (8, False), (64, True)])
def test_generic_matches_hf_olmoe(T, norm):
    from transformers import OlmoeConfig
    from transformers.models.olmoe.modeling_olmoe import OlmoeSparseMoeBlock

    E, H, I, k = 64, 512, 256, 8
    ex = _experts(E, H, I, 0.02, 1)
    g = torch.Generator().manual_seed(2 + T)
    wr = torch.randn((E, H), generator=g).to(bf16)
    h = torch.randn((T, H), generator=g).to(bf16)
    cfg = OlmoeConfig(hidden_size=H, intermediate_size=I, num_experts=E, num_experts_per_tok=k, norm_topk_prob=norm)
    blk = OlmoeSparseMoeBlock(cfg).to(bf16)
    _load_experts(blk.experts, ex)
    with torch.no_grad():
        blk.gate.weight.copy_(wr)
        _, _, hf_idx = blk.gate(h)
        hf = blk(h[None])[0]
    idx, _ = om.route(h, wr, k, norm)
    assert _same_routes(idx, hf_idx)
    assert _pinned(om.moe_layer(h, wr, None, ex, k, norm, residual=False, hf_rounding=True), hf, T)
    ours = om.moe_layer(h, wr, None, ex, k, norm, residual=False)
    err = om.rel_l2(ours, hf)
    assert err < TOL, err


@pytest.mark.parametrize("T", [1, 8, 64])
def test_qwen35_matches_hf_qwen3_5_moe(T):
    from transformers.models.qwen3_5_moe import configuration_qwen3_5_moe as qc
    from transformers.models.qwen3_5_moe import modeling_qwen3_5_moe as qm

    E, H, I, k = 64, 512, 256, 8
    ex = _experts(E + 1, H, I, 0.02, 3)
    shared = ex.pop()
    g = torch.Generator().manual_seed(4 + T)
    wr = torch.randn((E, H), generator=g).to(bf16)
    wsg = (torch.randn(H, generator=g) * 0.05).to(bf16)
    h = torch.randn((T, H), generator=g).to(bf16)
    cfg = qc.Qwen3_5MoeTextConfig(hidden_size=H, moe_intermediate_size=I, shared_expert_intermediate_size=I,
                                  num_experts=E, num_experts_per_tok=k)
    blk = qm.Qwen3_5MoeSparseMoeBlock(cfg).to(bf16)
    _load_experts(blk.experts, ex)
    _mlp(blk.shared_expert, shared)
    with torch.no_grad():
        blk.gate.weight.copy_(wr)
        blk.shared_expert_gate.weight.copy_(wsg[None])
        _, _, hf_idx = blk.gate(h)
        hf = blk(h[None])[0]
    idx, _ = om.route(h, wr, k, True, "qwen35")
    assert _same_routes(idx, hf_idx)
    kw = dict(residual=False, family="qwen35", shared=shared, shared_gate_w=wsg)
    assert _pinned(om.moe_layer(h, wr, None, ex, k, hf_rounding=True, **kw), hf, T)
    ours = om.moe_layer(h, wr, None, ex, k, **kw)
    err = om.rel_l2(ours, hf)
    assert err < TOL, err


def test_qwen35_zero_centred_norm_matches_hf():
    from transformers.models.qwen3_5_moe import modeling_qwen3_5_moe as qm

    g = torch.Generator().manual_seed(5)
    x = torch.randn((4, 512), generator=g).to(bf16)
    w = (0.1 * torch.randn(512, generator=g)).to(bf16)
    n = qm.Qwen3_5MoeRMSNorm(512, eps=1e-6)
    with torch.no_grad():
        n.weight.copy_(w.float())
        hf = n(x)
    assert torch.equal(om.rms_norm(x, w, 1e-6, plus_one=True), hf)


@pytest.mark.parametrize("T,norm", [(1, True), (8, True), (64, False)])
def test_glm_matches_hf_glm_moe_dsa(T, norm):
    from transformers import GlmMoeDsaConfig
    import transformers.models.glm_moe_dsa.modeling_glm_moe_dsa as gm

    E, H, I, k, scale = 64, 512, 256, 8, 2.5
    ex = _experts(E + 1, H, I, 0.02, 6)
    shared = ex.pop()
    g = torch.Generator().manual_seed(7 + T)
    wr = (torch.randn((E, H), generator=g) * 0.3).to(bf16)
    bias = torch.randn(E, generator=g) * 0.5
    h = torch.randn((T, H), generator=g).to(bf16)
    cfg = GlmMoeDsaConfig(vocab_size=64, hidden_size=H, intermediate_size=I, moe_intermediate_size=I,
                          num_hidden_layers=1, first_k_dense_replace=0, num_attention_heads=4,
                          num_key_value_heads=4, n_shared_experts=1, n_routed_experts=E, num_experts_per_tok=k,
                          n_group=1, topk_group=1, norm_topk_prob=norm, routed_scaling_factor=scale,
                          kv_lora_rank=16, q_lora_rank=32, qk_rope_head_dim=8, qk_nope_head_dim=8, v_head_dim=16,
                          index_topk=8, indexer_types=["full"])
    blk = gm.GlmMoeDsaMoE(cfg).to(bf16)
    _load_experts(blk.experts, ex)
    _mlp(blk.shared_experts, shared)
    with torch.no_grad():
        blk.gate.weight.copy_(wr)
        blk.gate.e_score_correction_bias = bias.clone()  # fp32, as checkpoints keep it
        hf_idx, _ = blk.route_tokens_to_experts(blk.gate(h))
        hf = blk(h[None])[0]
    idx, _ = om.route(h, wr, k, norm, "glm", bias, scale)
    assert _same_routes(idx, hf_idx)
    kw = dict(residual=False, family="glm", shared=shared, bias=bias, routed_scale=scale)
    assert _pinned(om.moe_layer(h, wr, None, ex, k, norm, hf_rounding=True, **kw), hf, T)
    ours = om.moe_layer(h, wr, None, ex, k, norm, **kw)
    err = om.rel_l2(ours, hf)
    assert err < TOL, err
