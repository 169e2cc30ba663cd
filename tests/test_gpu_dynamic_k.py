"""Dynamic K and router statistics on the GPU against the CPU oracle (model/layer.rs:947-1011,
2302-2334; config.rs:86-106, 468-483).

A tiny Qwen3-shaped K-quant model (8 layers, 32 experts, top-8) with router weights scaled up so
the routing entropy, and so K, varies by layer and token.  Both sides run one token per call.  Each
step must give the oracle's per-layer entropy (within 1e-6), K and routed experts, logits within
1e-3, and the greedy token; with layer_adaptive the K ranges follow the depth tiers.
"""
from dataclasses import replace

import numpy as np
import pytest

from moe_stream_b200 import gguf as G
from moe_stream_b200 import synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

SPEC = replace(synth.TINY_QWEN3, name="tiny-qwen3-dk", layers=8, experts=32, top_k=8)


def rel_err(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
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
def model_path(tmp_path_factory):
    m = synth.build_model(SPEC, seed=3)
    for name, t in list(m.tensors.items()):
        if name.endswith("ffn_gate_inp.weight"):
            m.add(name, t.qtype, t.shape, (t.data.view(np.float32) * np.float32(8.0)).astype(np.float32))
    p = str(tmp_path_factory.mktemp("dkg") / "m.gguf")
    G.write_gguf(p, m)
    return p


@pytest.mark.parametrize("adaptive", [False, True])
def test_dynamic_k_matches_oracle(ctx, orc, model_path, adaptive):
    from moe_stream_b200.engine import Engine
    L, E, K = SPEC.layers, SPEC.experts, SPEC.top_k
    eng = Engine.open(model_path, max_seq_len=64, ctx=ctx)
    eng.set_dynamic_k(True, 1, K, adaptive)
    om = orc.Model(model_path, max_seq_len=64)
    om.set_dynamic_k(True, 1, K, adaptive)
    tokens = list(synth.prompt_ids(SPEC, 6, seed=1))
    seen_k = set()
    for step in range(16):
        t = tokens[step]
        got = eng.forward([t])
        want = om.forward(np.array([t], np.int32))
        g_ent, g_k = eng.router_stats()
        w_ent, w_k = om.router_stats(L)
        assert g_k.tolist() == w_k.tolist(), f"step {step}"
        assert np.abs(g_ent - w_ent).max() <= 1e-6 * max(1.0, float(np.abs(w_ent).max()))
        w_idx, _ = om.last_routing(L, K)
        for li in range(L):
            gi, gw = eng.last_routing(li)
            assert gi.tolist() == w_idx[li].tolist(), f"step {step} layer {li}"
            assert (gw[g_k[li]:] == 0).all()
        assert rel_err(got, want) < 1e-3
        assert int(np.argmax(got)) == int(np.argmax(want))
        seen_k.update(g_k.tolist())
        if step + 1 >= len(tokens):
            tokens.append(int(np.argmax(want)))
    assert len(seen_k) >= 3   # K really varied
    eng.close()
    om.close()


def test_router_stats_without_dynamic_k(ctx, orc, model_path):
    from moe_stream_b200.engine import Engine
    eng = Engine.open(model_path, max_seq_len=16, ctx=ctx)
    eng.set_router_stats(True)
    eng.forward([3])
    ent, k = eng.router_stats()
    om = orc.Model(model_path, max_seq_len=16)
    om.forward(np.array([3], np.int32))
    w_ent, _ = om.router_stats(SPEC.layers)
    assert (k == SPEC.top_k).all()
    assert np.abs(ent - w_ent).max() <= 1e-6 * max(1.0, float(np.abs(w_ent).max()))
    eng.close()
    om.close()


def test_router_totals_accumulate_on_device(ctx, model_path):
    """RoutingStatsCollector / EntropyProfiler totals kept by the router on the device equal the
    per-step routing and entropy read back after every step; re-enabling starts from zero"""
    from moe_stream_b200.engine import Engine
    L, E, K = SPEC.layers, SPEC.experts, SPEC.top_k
    eng = Engine.open(model_path, max_seq_len=64, ctx=ctx)
    eng.set_dynamic_k(True, 1, K)
    eng.set_router_stats(True)
    cnt = np.zeros((L, E), np.uint64)
    wsum = np.zeros((L, E), np.float64)
    ents = []
    tokens = list(synth.prompt_ids(SPEC, 12, seed=4))
    for t in tokens:
        eng.forward([t])
        e, k = eng.router_stats()
        ents.append(e)
        for li in range(L):
            gi, gw = eng.last_routing(li)
            for j in range(int(k[li])):
                cnt[li, gi[j]] += 1
                wsum[li, gi[j]] += float(gw[j])
    tot = eng.router_totals()
    assert tot["steps"] == len(tokens) and (tot["tokens"] == len(tokens)).all()
    assert np.array_equal(tot["counts"], cnt)
    assert np.array_equal(tot["weight_sums"], wsum)   # f64 sums in the same (step) order
    assert np.array_equal(tot["entropy_log"], np.stack(ents))
    assert np.allclose(tot["importance"], cnt / len(tokens) * np.where(cnt > 0, wsum / np.maximum(cnt, 1), 0))
    eng.set_router_stats(True)
    assert eng.router_totals()["steps"] == 0
    eng.close()
