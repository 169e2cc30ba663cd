"""GPU parity of the DeltaNet hybrid model step (Qwen3-Next shape, configs[3]) through the C ABI.

A seeded tiny Qwen3-Next-shaped model (moe_stream_b200.synth.TINY_QWEN3_NEXT: Gated DeltaNet layers
with gated attention every 4th layer, head_dim 256 with rotary 0.25, 64 experts top-10 and a shared
expert) against the CPU oracle's fixture tests/golden/tiny_qwen3_next.npz.  Layer dispatch follows
config.rs:446-458 and model/layer.rs:393-503.  Tolerances: per-layer residual stream and logits within
1e-3 relative (DeltaNet, the shared expert and head_dim-256 attention accumulate in f32 in their own
order); routed experts exact; greedy tokens identical.  The oracle's smallest top-2 logit margin over
these 24 tokens is 0.66 % relative, far above the f32 differences, so token equality is a real check.
"""
import os

import numpy as np
import pytest

from moe_stream_b200 import synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden", "tiny_qwen3_next.npz")
REL_TOL = 1e-3
SEED = 11


def rel_err(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-30))


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from moe_stream_b200.engine import Context
    c = Context(0)
    yield c
    c.close()


@pytest.fixture(scope="module")
def hybrid_path(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("hyb") / "tiny_qwen3_next.gguf")
    synth.write_model(p, synth.TINY_QWEN3_NEXT, seed=SEED)
    return p


def test_hybrid_model_layers_routing_and_tokens(ctx, hybrid_path):
    from moe_stream_b200.engine import Engine
    spec = synth.TINY_QWEN3_NEXT
    f = np.load(GOLD)
    eng = Engine.open(hybrid_path, max_seq_len=64, ctx=ctx)
    c = eng.config
    assert (c.attn_interval, c.ssm_groups, c.ssm_state, c.ssm_dt_rank, c.ssm_inner, c.ssm_conv) == \
        (4, spec.ssm_groups, spec.ssm_state, spec.ssm_dt_rank, spec.ssm_inner, spec.ssm_conv)
    assert c.rot_dim == 64
    eng.set_trace(True)
    logits = eng.forward(f["prompt"])
    assert rel_err(logits, f["logits"]) < REL_TOL
    hid, _ = eng.layer_trace()
    for li in range(spec.layers):
        assert rel_err(hid[li], f["layer_hidden"][li]) < REL_TOL, f"layer {li}"
        gi, _ = eng.last_routing(li)
        assert sorted(gi.tolist()) == sorted(f["routing_idx"][li].tolist()), f"layer {li} routing"
    eng.set_trace(False)
    tokens = eng.generate(f["prompt"], len(f["tokens"]))
    assert tokens == f["tokens"].tolist()
    # the same continuation without the captured graph, and after clear_cache (DeltaNet states reset)
    eng.set_graph(False)
    assert eng.generate(f["prompt"], 8) == f["tokens"][:8].tolist()
    eng.close()


def test_hybrid_model_in_memory_upload(ctx):
    """ms_model_create + ms_model_set_tensor (split ssm_beta / ssm_alpha rows instead of ssm_ba)"""
    from moe_stream_b200 import gguf as G
    from moe_stream_b200.engine import Engine
    spec = synth.TINY_QWEN3_NEXT
    f = np.load(GOLD)
    m = synth.build_model(spec, seed=SEED)
    nv, H = spec.ssm_dt_rank, spec.hidden
    for li in range(spec.layers):
        name = f"blk.{li}.ssm_ba.weight"
        if name in m.tensors:
            t = m.tensors.pop(name)
            rb = t.raw().size // (2 * nv)
            m.add(f"blk.{li}.ssm_beta.weight", t.qtype, (nv, H), t.raw()[:nv * rb])
            m.add(f"blk.{li}.ssm_alpha.weight", t.qtype, (nv, H), t.raw()[nv * rb:])
    eng = Engine.from_model(m, max_seq_len=64, ctx=ctx)
    assert eng.generate(f["prompt"], 12) == f["tokens"][:12].tolist()
    eng.close()
