"""Dynamic K and router statistics in the CPU oracle (model/layer.rs:947-1011, 2302-2334;
config.rs:86-106, 183-192, 468-483) against a float64 numpy restatement of the same rules:
entropy of softmax(router logits) per layer, K = round(k_min + clamp(H / ln E, 0, 1) (k_max - k_min)),
top-K routing with the weights renormalised over the K selected, and the depth tiers of
LayerTierConfig::default_for_k when layer_adaptive is set."""
import numpy as np
import pytest

from moe_stream_b200 import synth


def tier_range(li, layers, k_min, k_max, adaptive):
    if not adaptive:
        return k_min, k_max
    two_thirds = min(max(k_max * 2 // 3, 4), k_max)
    depth = np.float32(li) / np.float32(layers)
    if depth < np.float32(0.15):
        return k_max, k_max
    if depth < np.float32(0.85):
        return min(4, k_max), two_thirds
    return two_thirds, k_max


def sharp_router_model(seed=21, scale=8.0):
    """the tiny hybrid with router weights scaled up, so the routing entropy (and K) varies"""
    from moe_stream_b200 import gguf as G
    m = synth.build_model(synth.TINY_QWEN3_NEXT, seed=seed)
    for name, t in list(m.tensors.items()):
        if name.endswith("ffn_gate_inp.weight"):
            m.add(name, t.qtype, t.shape, (t.data.view(np.float32) * np.float32(scale)).astype(np.float32))
    return m


@pytest.fixture(scope="module")
def model_path(tmp_path_factory):
    from moe_stream_b200 import gguf as G
    p = str(tmp_path_factory.mktemp("dk") / "m.gguf")
    G.write_gguf(p, sharp_router_model())
    return p


@pytest.mark.parametrize("k_min,k_max,adaptive", [(2, 10, False), (3, 8, False), (2, 10, True)])
def test_dynamic_k_entropy_and_routing(orc, model_path, k_min, k_max, adaptive):
    spec = synth.TINY_QWEN3_NEXT
    E, L, K = spec.experts, spec.layers, spec.top_k
    om = orc.Model(model_path, max_seq_len=16)
    om.set_dynamic_k(True, k_min, k_max, adaptive)
    prompt = synth.prompt_ids(spec, 3, seed=2)
    for t in prompt:   # one token per call: K is per token
        om.forward(np.array([t], np.int32))
        ent, ks = om.router_stats(L)
        _, logits = om.layer_trace(L, E)
        idx, w = om.last_routing(L, K)
        for li in range(L):
            lg = logits[li].astype(np.float64)
            p = np.exp(lg - lg.max())
            p /= p.sum()
            h = -(p[p > 0] * np.log(p[p > 0])).sum()
            assert abs(ent[li] - h) <= 1e-5 * max(1.0, h)
            lo, hi = tier_range(li, L, k_min, k_max, adaptive)
            kf = lo + min(max(h / np.log(E), 0.0), 1.0) * (hi - lo)
            if abs(kf - np.floor(kf) - 0.5) > 1e-4:   # not on a rounding boundary
                assert ks[li] == min(max(int(np.floor(kf + 0.5)), lo), hi)
            k = ks[li]
            assert lo <= k <= hi
            order = np.argsort(-p, kind="stable")[:k]
            assert idx[li, :k].tolist() == order.tolist()
            assert (idx[li, k:] == E).all() and (w[li, k:] == 0).all()
            np.testing.assert_allclose(w[li, :k], p[order] / p[order].sum(), rtol=1e-5)
    om.close()


def test_dynamic_k_disabled_keeps_top_k(orc, model_path):
    spec = synth.TINY_QWEN3_NEXT
    om = orc.Model(model_path, max_seq_len=16)
    om.set_dynamic_k(True, 2, 10)
    om.set_dynamic_k(False)
    om.forward(np.array([5], np.int32))
    _, ks = om.router_stats(spec.layers)
    assert (ks == spec.top_k).all()
    with pytest.raises(ValueError):
        om.set_dynamic_k(True, 3, spec.top_k + 1)
    om.close()
