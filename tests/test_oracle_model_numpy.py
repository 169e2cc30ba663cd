"""One token through the oracle's GPT-OSS-shaped model (the benchmark's architecture: sinks, sliding
window on even layers, biases, softmax over the selected top-k, OAI SwiGLU, f16 embedding and LM
head) and its Qwen3-shaped model (QK-norm, softmax over all experts then renormalised top-k, SiLU,
Q4_K / Q6_K experts) against a float64 numpy composition of the reference's steps (engine.rs:1869-2006,
layer.rs:393-503), per layer within 1e-4.  The oracle runs its projections in exact-f32 mode here, so
the comparison measures the model wiring rather than Q8_0 activation rounding."""
import numpy as np

from moe_stream_b200 import gguf as G
from moe_stream_b200 import synth

from .moe_ref import moe_with_routing
from .test_oracle_attention import _attn_np


import pytest


@pytest.mark.parametrize("spec", [synth.TINY_GPT_OSS, synth.TINY_QWEN3], ids=["gpt-oss", "qwen3"])
def test_model_one_token_matches_numpy(orc, tmp_path, spec):
    oai = spec.arch == "gpt-oss"
    m = synth.build_model(spec, seed=13)
    path = str(tmp_path / "g.gguf")
    G.write_gguf(path, m)
    T = m.tensors
    H, E, K = spec.hidden, spec.experts, spec.top_k
    token = 77
    om = orc.Model(path, max_seq_len=8, attn_mode=0)
    o_logits = om.forward(np.array([token], np.int32))
    o_hid, o_lg = om.layer_trace(spec.layers, E)
    o_idx, o_w = om.last_routing(spec.layers, K)
    om.close()
    h = T["token_embd.weight"].data.reshape(spec.vocab, H)[token].astype(np.float64)
    for li in range(spec.layers):
        p = f"blk.{li}."
        f32 = lambda n: T[p + n].data.astype(np.float32) if p + n in T else None
        d = dict(hidden=H, heads=spec.heads, kv_heads=spec.kv_heads, head_dim=spec.head_dim, rot_dim=spec.head_dim,
                 eps=spec.eps, rope_theta=spec.rope_theta, window=spec.sliding_window if li % 2 == 0 else 0,
                 attn_norm=f32("attn_norm.weight"), wq=T[p + "attn_q.weight"].raw(), wk=T[p + "attn_k.weight"].raw(),
                 wv=T[p + "attn_v.weight"].raw(), wo=T[p + "attn_output.weight"].raw(), bq=f32("attn_q.bias"),
                 bk=f32("attn_k.bias"), bv=f32("attn_v.bias"), bo=f32("attn_output.bias"),
                 sinks=f32("attn_sinks.weight"), q_norm=f32("attn_q_norm.weight"), k_norm=f32("attn_k_norm.weight"))
        h = _attn_np(orc, d, h, [], [], 0)
        x = h / np.sqrt((h * h).mean() + spec.eps) * f32("post_attention_norm.weight" if oai else "ffn_norm.weight")
        logits = f32("ffn_gate_inp.weight").reshape(E, H).astype(np.float64) @ x
        if f32("ffn_gate_inp.bias") is not None:
            logits = logits + f32("ffn_gate_inp.bias")
        assert np.abs(o_lg[li] - logits).max() / np.abs(logits).max() < 1e-5
        srt = np.sort(logits)[::-1]
        assert srt[K - 1] - srt[K] > 1e-5, "seed has a near-tie at the top-k boundary"
        order = np.argsort(-logits, kind="stable")[:K]
        assert order.tolist() == o_idx[li].tolist()
        if oai:   # softmax over the selected logits (layer.rs:2361-2372)
            w = np.exp(logits[order] - logits[order].max())
        else:     # softmax over all, then renormalised over the selected (layer.rs:2374-2394)
            w = np.exp(logits - logits.max())[order]
        w /= w.sum()
        np.testing.assert_allclose(o_w[li], w, rtol=1e-5)
        L = dict(hidden=H, inter=spec.inter, n_experts=E, top_k=K, gate_q=spec.expert_gate_q, up_q=spec.expert_gate_q,
                 down_q=spec.expert_down_q, gate=T[p + "ffn_gate_exps.weight"].raw(),
                 up=T[p + "ffn_up_exps.weight"].raw(), down=T[p + "ffn_down_exps.weight"].raw(),
                 gate_bias=f32("ffn_gate_exps.bias"), up_bias=f32("ffn_up_exps.bias"),
                 down_bias=f32("ffn_down_exps.bias"), oai_swiglu=int(oai))
        h = h + moe_with_routing(orc, L, x, order, w)
        assert np.abs(o_hid[li] - h).max() / np.abs(h).max() < 1e-4, f"layer {li}"
    xf = h / np.sqrt((h * h).mean() + spec.eps) * T["output_norm.weight"].data
    logits = T["output.weight"].data.reshape(spec.vocab, H).astype(np.float64) @ xf
    assert np.abs(o_logits - logits).max() / np.abs(logits).max() < 1e-4
    assert int(np.argmax(o_logits)) == int(np.argmax(logits))


@pytest.mark.parametrize("spec", [synth.TINY_GPT_OSS, synth.TINY_QWEN3, synth.TINY_QWEN3_NEXT],
                         ids=["gpt-oss", "qwen3", "qwen3-next"])
def test_multi_token_forward_equals_token_by_token(orc, tmp_path, spec):
    """the oracle's prompt forward (causal attention over the call's positions, layer.rs:393-503 with
    seq_len > 1; DeltaNet token by token) gives the logits and per-layer residuals of feeding the same
    tokens one call at a time -- the reference the batched GPU prefill is compared with"""
    path = str(tmp_path / "m.gguf")
    synth.write_model(path, spec, seed=17)
    prompt = synth.prompt_ids(spec, 11, seed=17)
    a = orc.Model(path, max_seq_len=32)
    la = a.forward(prompt)
    ha, _ = a.layer_trace(spec.layers, spec.experts)
    b = orc.Model(path, max_seq_len=32)
    for t in prompt:
        lb = b.forward(np.array([t], np.int32))
    hb, _ = b.layer_trace(spec.layers, spec.experts)
    assert np.abs(la - lb).max() / np.abs(lb).max() < 1e-5
    assert np.abs(ha - hb).max() / np.abs(hb).max() < 1e-5
    a.close()
    b.close()
