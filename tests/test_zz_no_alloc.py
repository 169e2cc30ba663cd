"""The allocation-free MoE entry point (ms_moe_mxfp4_decode_noalloc).

It serves callers that cannot allocate device memory while they run the MoE step (a fixed
pool owns the memory budget, or the step runs where cudaMalloc is not allowed).  Its output
must match the regular entry point (ms_moe_mxfp4_decode), which allocates its scratch from
the context, on consecutive calls that reuse the fixed scratch array.  This file is collected
last so a failure here never hides another test's result.
"""
import numpy as np
import pytest

from moe_stream_b200 import synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

REL_TOL = 1e-3


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.fixture(scope="module")
def setup():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from moe_stream_b200.engine import Context
    ctx = Context(0)
    ctx.set_stream(torch.cuda.current_stream())
    spec = synth.GPT_OSS_MOE_LAYER
    m = synth.build_model(spec, seed=21, only=lambda n: "exps" in n)
    pad = np.zeros(16 * 4352, np.uint8)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    t = lambda n: m.tensors["blk.0." + n]
    W = dict(gate=d(np.concatenate([t("ffn_gate_exps.weight").raw(), pad])),
             up=d(np.concatenate([t("ffn_up_exps.weight").raw(), pad])),
             down=d(np.concatenate([t("ffn_down_exps.weight").raw(), pad])),
             gate_b=d(t("ffn_gate_exps.bias").data), up_b=d(t("ffn_up_exps.bias").data),
             down_b=d(t("ffn_down_exps.bias").data))
    yield ctx, spec, W
    ctx.close()


def _run(ctx, spec, W, fn, x, idx, wts, h0):
    h = h0.clone()
    fn(W["gate"], W["up"], W["down"], W["gate_b"], W["up_b"], W["down_b"], spec.hidden, spec.inter,
       spec.experts, spec.top_k, 0, x, idx, wts, h)
    ctx.sync()
    return h.cpu().numpy()


def test_noalloc_matches_regular_entry_point_on_consecutive_calls(setup):
    ctx, spec, W = setup
    rng = np.random.default_rng(5)
    for call in range(2):   # the second call runs on the array the first call left behind
        x = torch.from_numpy(rng.standard_normal(spec.hidden).astype(np.float32)).cuda()
        h0 = torch.from_numpy(rng.standard_normal(spec.hidden).astype(np.float32)).cuda()
        idx = torch.from_numpy(rng.permutation(spec.experts)[:spec.top_k].astype(np.int32)).cuda()
        wts = torch.softmax(torch.from_numpy(rng.standard_normal(spec.top_k).astype(np.float32)), 0).cuda()
        want = _run(ctx, spec, W, ctx.moe_mxfp4_decode, x, idx, wts, h0)
        got = _run(ctx, spec, W, ctx.moe_mxfp4_decode_noalloc, x, idx, wts, h0)
        assert _rel(got - h0.cpu().numpy(), want - h0.cpu().numpy()) < REL_TOL, f"call {call}"


def test_noalloc_rejects_sizes_beyond_its_scratch(setup):
    ctx, spec, W = setup
    from moe_stream_b200._lib import MsError
    x = torch.zeros(8192, device="cuda")
    idx = torch.zeros(4, dtype=torch.int32, device="cuda")
    wts = torch.zeros(4, device="cuda")
    with pytest.raises(MsError) as ei:
        ctx.moe_mxfp4_decode_noalloc(W["gate"], W["up"], W["down"], None, None, None, 8192, 2880, 32, 4, 0,
                                     x, idx, wts, x)
    assert ei.value.status == 7 and "exceed the fixed scratch" in str(ei.value)


def test_noalloc_at_its_size_limits(setup):
    """top_k 16 with hidden = inter = 4096: the activation and partial slices fill the array"""
    ctx, _, _ = setup
    H = I = 4096
    E, K = 16, 16
    rng = np.random.default_rng(8)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    pad = np.zeros(16 * 4352, np.uint8)
    gate = d(np.concatenate([synth.rand_mxfp4(rng, E * I * H), pad]))
    up = d(np.concatenate([synth.rand_mxfp4(rng, E * I * H), pad]))
    down = d(np.concatenate([synth.rand_mxfp4(rng, E * H * I), pad]))
    bias = [d((rng.standard_normal(E * n) * 0.01).astype(np.float32)) for n in (I, I, H)]
    for call in range(2):
        x = d(rng.standard_normal(H).astype(np.float32))
        h0 = d(rng.standard_normal(H).astype(np.float32))
        idx = d(rng.permutation(E)[:K].astype(np.int32))
        wts = torch.softmax(torch.from_numpy(rng.standard_normal(K).astype(np.float32)), 0).cuda()
        outs = []
        for fn in (ctx.moe_mxfp4_decode, ctx.moe_mxfp4_decode_noalloc):
            h = h0.clone()
            fn(gate, up, down, bias[0], bias[1], bias[2], H, I, E, K, 0, x, idx, wts, h)
            ctx.sync()
            outs.append(h.cpu().numpy() - h0.cpu().numpy())
        assert _rel(outs[1], outs[0]) < REL_TOL, f"call {call}"
