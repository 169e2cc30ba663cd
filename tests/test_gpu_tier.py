"""Host-tier expert streaming on the GPU (the reference's SSD-streaming mode with its per-layer expert
LRU: gguf/reader.rs:631-858, model/layer.rs:1146-1152, 1777-1784, model/cache.rs:84-158).

The expert stacks stay in pinned host memory and HBM holds a few expert slots per layer.  The same
order-independent expert kernels run on the slots, so the model must produce the same bits as with
HBM-resident experts: identical greedy tokens and bit-identical logits.  The slot hits and misses must
equal a replay of the LRU policy (empty slot first, else the least recently used slot not routed in
the current step) over the routed experts of every step.
"""
import numpy as np
import pytest

from moe_stream_b200 import synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from moe_stream_b200.engine import Context
    c = Context(0)
    yield c
    c.close()


def lru_replay(routes, slots):
    """hits, misses of the slot policy over routes[step][layer] = routed experts in slot order"""
    n_layers = len(routes[0])
    cache = [[-1] * slots for _ in range(n_layers)]
    used = [[0] * slots for _ in range(n_layers)]
    now = hits = misses = 0
    for step in routes:
        for li, experts in enumerate(step):
            now += 1
            sl, us = cache[li], used[li]
            missing = []
            for e in experts:
                if e in sl:
                    us[sl.index(e)] = now
                    hits += 1
                else:
                    missing.append(e)
            for e in missing:
                if -1 in sl:
                    j = sl.index(-1)
                else:
                    cand = [j for j in range(slots) if us[j] != now]
                    j = min(cand, key=lambda q: (us[q], q))
                sl[j], us[j] = e, now
                misses += 1
    return hits, misses


@pytest.mark.parametrize("spec_name,slots", [("tiny-qwen3", 6), ("tiny-qwen3-next", 12)])
def test_host_tier_matches_resident_experts(ctx, tmp_path, spec_name, slots):
    from moe_stream_b200.engine import Engine
    spec = synth.PRESETS[spec_name]
    path = str(tmp_path / "m.gguf")
    synth.write_model(path, spec, seed=5)
    prompt = synth.prompt_ids(spec, 6, seed=5)
    n_new = 16
    res = Engine.open(path, max_seq_len=64, ctx=ctx)
    res.set_prefill(0)   # one decode step per prompt token, as the tiered model runs its prompt
    want = res.generate(prompt, n_new)
    res.clear_cache()
    want_logits = res.forward(prompt)
    # the routed experts of every step the tiered run will take (one step per position)
    res.clear_cache()
    routes = []
    for t in list(prompt) + want[:-1]:
        res.forward([t])
        routes.append([res.last_routing(li)[0].tolist() for li in range(spec.layers)])
    res.close()

    tier = Engine.open(path, max_seq_len=64, ctx=ctx, expert_slots=slots)
    assert tier.generate(prompt, n_new) == want
    tier.clear_cache()
    got_logits = tier.forward(prompt)
    assert np.array_equal(got_logits.view(np.uint32), want_logits.view(np.uint32))
    hits, misses = tier.expert_tier_stats()
    want_hits, want_misses = lru_replay(routes + routes[:len(prompt)], slots)
    assert (hits, misses) == (want_hits, want_misses)
    assert hits > 0 and misses > spec.layers * slots   # the cache both hit and evicted
    tier.close()


def test_host_tier_refusals(ctx, tmp_path):
    """MXFP4 experts (tensor-core tiles) have no host tier; slots below top_k are refused"""
    from moe_stream_b200.engine import Engine
    from moe_stream_b200._lib import MsError
    path = str(tmp_path / "g.gguf")
    synth.write_model(path, synth.TINY_GPT_OSS, seed=1)
    with pytest.raises(MsError):
        Engine.open(path, max_seq_len=32, ctx=ctx, expert_slots=8)
    qpath = str(tmp_path / "q.gguf")
    synth.write_model(qpath, synth.TINY_QWEN3, seed=1)
    with pytest.raises(MsError):
        Engine.open(qpath, max_seq_len=32, ctx=ctx, expert_slots=synth.TINY_QWEN3.top_k - 1)
