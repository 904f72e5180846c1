"""Pins the fp32 gpt-oss decoding restatement (tests/_gptoss_ref.py), which the GPU decoder tests compare
against, to transformers' own GptOssForCausalLM (eager attention, fp32, CPU) on a tiny config whose
sliding window (4) is shorter than the sequence, and checks the rotary tables the decoder feeds its
kernel against HF's rotary on a head."""

import torch

from _gptoss_ref import RefGptOss, rotate


def _tiny():
    from wisp.gptoss_decoder import GptOssDecoderConfig

    return GptOssDecoderConfig(vocab=97, hidden=64, layers=3, heads=4, kv_heads=2, head_dim=16, experts=8, top_k=2, inter=64,
                               window=4)


def _hf_params(model, cfg):
    m = model.model
    p = dict(embed=m.embed_tokens.weight.detach(), lm_head=model.lm_head.weight.detach(), final_norm=m.norm.weight.detach(),
             layers=[])
    for ly in m.layers:
        a, e = ly.self_attn, ly.mlp.experts
        p["layers"].append(dict(
            in_norm=ly.input_layernorm.weight, post_norm=ly.post_attention_layernorm.weight,
            wq=a.q_proj.weight, bq=a.q_proj.bias, wk=a.k_proj.weight, bk=a.k_proj.bias, wv=a.v_proj.weight, bv=a.v_proj.bias,
            wo=a.o_proj.weight, bo=a.o_proj.bias, sinks=a.sinks, router=ly.mlp.router.weight, router_b=ly.mlp.router.bias,
            gate_up=e.gate_up_proj, gub=e.gate_up_proj_bias, down=e.down_proj, db=e.down_proj_bias))
        p["layers"][-1] = {k: v.detach() for k, v in p["layers"][-1].items()}
    return p


@torch.no_grad()
def test_reference_matches_transformers():
    from transformers import GptOssForCausalLM

    from wisp.gptoss_decoder import gptoss_rotary_half

    cfg = _tiny()
    hc = cfg.hf(max_positions=64)
    hc._attn_implementation = "eager"
    hc.initializer_range = 0.2  # larger than the default so attention and routing are not flat
    torch.manual_seed(0)
    model = GptOssForCausalLM(hc).float().eval()
    for ly in model.model.layers:  # HF initialises biases and sinks to zero / small: give them weight
        for prm in (ly.self_attn.sinks, ly.self_attn.q_proj.bias, ly.mlp.router.bias, ly.mlp.experts.gate_up_proj_bias,
                    ly.mlp.experts.down_proj_bias):
            prm.normal_(0, 0.5)
    T, B = 10, 2
    ids = torch.randint(0, cfg.vocab, (B, T))
    want = model(ids).logits  # full-sequence forward: causal + sliding-window masks
    cos, sin = gptoss_rotary_half(cfg, 64, "cpu")
    ref = RefGptOss(_hf_params(model, cfg), cfg, cos, sin, B, 64)
    for t in range(T):
        got, _, _ = ref.step(ids[:, t], torch.full((B,), t))
        assert torch.allclose(got, want[:, t], atol=1e-4, rtol=1e-4), (t, (got - want[:, t]).abs().max())


def test_rotary_tables_match_transformers():
    from transformers.models.gpt_oss.modeling_gpt_oss import apply_rotary_pos_emb

    from wisp.gptoss_decoder import GptOssDecoderConfig, gptoss_rotary_half, gptoss_rotary_tables

    cfg = GptOssDecoderConfig()  # the real gpt-oss-20b rotary: YaRN factor 32, theta 150000, head 64
    cos, sin = gptoss_rotary_half(cfg, 300, "cpu")
    q = torch.randn(1, 2, 300, 64)
    want, _ = apply_rotary_pos_emb(q, q, cos[None], sin[None])
    assert torch.allclose(rotate(q, cos, sin), want, atol=1e-6)
    cf, sf = gptoss_rotary_tables(cfg, 300, "cpu")  # rotate-half form the kernel evaluates
    x = q[0, 0]
    rh = torch.cat([-x[:, 32:], x[:, :32]], -1)
    assert (x * cf.float() + rh * sf.float() - want[0, 0]).abs().max() < 0.05 * want.abs().max()
