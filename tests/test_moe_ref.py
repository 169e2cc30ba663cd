"""The float64 MoE restatement used by GPU tests with supplied routings agrees with the oracle's
layer when given the oracle's own routing."""
import numpy as np

from moe_stream_b200 import synth

from .moe_ref import moe_with_routing


def test_moe_ref_matches_oracle(orc):
    spec = synth.TINY_GPT_OSS
    m = synth.build_model(spec, 3)
    p = "blk.0."
    t = lambda n: m.tensors[p + n].raw()
    f = lambda n: m.tensors[p + n].data.astype(np.float32)
    L = dict(hidden=spec.hidden, inter=spec.inter, n_experts=spec.experts, top_k=spec.top_k,
             gate_q=spec.expert_gate_q, up_q=spec.expert_gate_q, down_q=spec.expert_down_q,
             gate=t("ffn_gate_exps.weight"), up=t("ffn_up_exps.weight"), down=t("ffn_down_exps.weight"),
             gate_bias=f("ffn_gate_exps.bias"), up_bias=f("ffn_up_exps.bias"),
             down_bias=f("ffn_down_exps.bias"), router_w=f("ffn_gate_inp.weight"),
             router_b=f("ffn_gate_inp.bias"), oai_swiglu=1, norm_topk_prob=1)
    x = synth.moe_layer_input(spec, seed=3) * 7.0
    want, idx, w = orc.moe_forward(L, x)
    got = moe_with_routing(orc, L, x, idx[0], w[0])
    assert np.abs(got - want[0]).max() / np.abs(want[0]).max() < 1e-5
