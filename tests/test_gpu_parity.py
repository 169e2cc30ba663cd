"""GPU parity of the CUDA path (through the C ABI) against the CPU oracle and golden fixtures.

Tolerances: block dequantization and routed expert indices are bit-exact; per-layer
outputs are within 1e-3 relative (max-abs error over max-abs reference) in f32
accumulation; greedy tokens are identical.
"""
import os

import numpy as np
import pytest

from moe_stream_b200 import gguf as G
from moe_stream_b200 import synth

from . import hybrid_synth as hs
from .moe_ref import moe_with_routing

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")
REL_TOL = 1e-3


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
    c.set_stream(torch.cuda.current_stream())
    yield c
    c.close()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def pad_rows(raw: np.ndarray, extra: int = 16 * 4352) -> np.ndarray:
    """streaming kernels may read up to one 16-row tile past the last row"""
    return np.concatenate([raw, np.zeros(extra, np.uint8)])


@pytest.mark.parametrize("key,qtype", [("mxfp4", G.MXFP4), ("q4_k", G.Q4_K), ("q6_k", G.Q6_K),
                                       ("q8_0", G.Q8_0), ("f16", G.F16)])
def test_dequant_bit_exact(ctx, key, qtype):
    f = np.load(os.path.join(GOLD, "dequant_kat.npz"))
    raw, want = f[f"{key}_raw"], f[f"{key}_out"]
    out = torch.empty(want.size, dtype=torch.float32, device="cuda")
    ctx.dequantize(qtype, dev(raw), want.size, out)
    ctx.sync()
    got = out.cpu().numpy()
    same = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
    assert same.all(), f"{(~same).sum()} mismatches"


def test_dequant_full_expert_matrix(ctx, orc):
    rng = np.random.default_rng(11)
    raw = synth.rand_mxfp4(rng, 2880 * 2880, 0, 255)
    out = torch.empty(2880 * 2880, dtype=torch.float32, device="cuda")
    ctx.dequantize(G.MXFP4, dev(raw), out.numel(), out)
    ctx.sync()
    want = orc.dequantize(G.MXFP4, raw, out.numel())
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("rows,cols", [(2880, 2880), (16, 64), (37, 2880), (5760, 2880)])
def test_mxfp4_gemv(ctx, orc, rows, cols):
    rng = np.random.default_rng(rows * 7 + cols)
    w = synth.rand_mxfp4(rng, rows * cols)
    x = rng.standard_normal(cols).astype(np.float32)
    b = (rng.standard_normal(rows) * 0.01).astype(np.float32)
    y = torch.empty(rows, dtype=torch.float32, device="cuda")
    ctx.gemv(G.MXFP4, dev(pad_rows(w)), rows, cols, dev(x), y, bias=dev(b))
    ctx.sync()
    want = orc.gemv(G.MXFP4, w, rows, cols, x) + b
    assert rel_err(y.cpu().numpy(), want) < 1e-5


def test_mxfp4_gemv_scale_extremes(ctx, orc):
    """activations spanning 2^-20..2^10 and e8m0 scales 100..140"""
    rng = np.random.default_rng(5)
    rows, cols = 64, 1024
    w = synth.rand_mxfp4(rng, rows * cols, 100, 140)
    x = (rng.standard_normal(cols) * np.exp2(rng.integers(-20, 10, cols))).astype(np.float32)
    y = torch.empty(rows, dtype=torch.float32, device="cuda")
    ctx.gemv(G.MXFP4, dev(pad_rows(w)), rows, cols, dev(x), y)
    ctx.sync()
    dense = orc.dequantize(G.MXFP4, w, rows * cols).reshape(rows, cols).astype(np.float64)
    assert rel_err(y.cpu().numpy(), dense @ x.astype(np.float64)) < 1e-5


@pytest.mark.parametrize("qtype,rows,cols", [(G.Q4_K, 768, 2048), (G.Q6_K, 2048, 768), (G.Q4_K, 16, 256),
                                             (G.Q6_K, 37, 512), (G.Q4_K, 512, 2048)])
def test_kquant_gemv(ctx, orc, qtype, rows, cols):
    rng = np.random.default_rng(rows * 3 + cols + qtype)
    w = synth.rand_q4_k(rng, rows * cols) if qtype == G.Q4_K else synth.rand_q6_k(rng, rows * cols)
    x = rng.standard_normal(cols).astype(np.float32)
    y = torch.empty(rows, dtype=torch.float32, device="cuda")
    ctx.gemv(qtype, dev(pad_rows(w)), rows, cols, dev(x), y)
    ctx.sync()
    dense = orc.dequantize(qtype, w, rows * cols).reshape(rows, cols).astype(np.float64)
    assert rel_err(y.cpu().numpy(), dense @ x.astype(np.float64)) < 1e-5


@pytest.mark.parametrize("rows,cols", [(5120, 2880), (2880, 4096), (64, 64), (13, 2048)])
def test_q8_0_gemv_activation_quantized(ctx, orc, rows, cols):
    rng = np.random.default_rng(rows + cols)
    w = synth.rand_q8_0(rng, rows * cols)
    x = rng.standard_normal(cols).astype(np.float32)
    y = torch.empty(rows, dtype=torch.float32, device="cuda")
    ctx.gemv(G.Q8_0, dev(pad_rows(w)), rows, cols, dev(x), y)
    ctx.sync()
    want = orc.q8_0_gemv(w, rows, cols, x, mode=1)   # candle QMatMul numerics
    assert rel_err(y.cpu().numpy(), want) < 1e-5


@pytest.mark.parametrize("rows,cols", [(1000, 2880), (4099, 2048)])
def test_f16_gemv(ctx, orc, rows, cols):
    rng = np.random.default_rng(rows)
    w = (rng.standard_normal(rows * cols) * 0.02).astype(np.float16)
    x = rng.standard_normal(cols).astype(np.float32)
    y = torch.empty(rows, dtype=torch.float32, device="cuda")
    ctx.gemv(G.F16, dev(w), rows, cols, dev(x), y)
    ctx.sync()
    want = orc.gemv(G.F16, w.view(np.uint8), rows, cols, x)
    assert rel_err(y.cpu().numpy(), want) < 1e-5


def test_rms_norm(ctx, orc):
    rng = np.random.default_rng(2)
    x = rng.standard_normal((3, 2880)).astype(np.float32) * 3
    w = (1 + 0.1 * rng.standard_normal(2880)).astype(np.float32)
    y = torch.empty_like(dev(x))
    ctx.rms_norm(dev(x), dev(w), y, 3, 2880, 1e-5)
    ctx.sync()
    assert rel_err(y.cpu().numpy(), orc.rms_norm(x, w, 1e-5)) < 1e-6


def _moe_layer_host(spec, seed):
    m = synth.build_model(spec, seed)
    p = "blk.0."
    t = lambda n: m.tensors[p + n].raw()
    f = lambda n: m.tensors[p + n].data.astype(np.float32)
    L = dict(hidden=spec.hidden, inter=spec.inter, n_experts=spec.experts, top_k=spec.top_k,
             gate_q=spec.expert_gate_q, up_q=spec.expert_gate_q, down_q=spec.expert_down_q,
             gate=t("ffn_gate_exps.weight"), up=t("ffn_up_exps.weight"), down=t("ffn_down_exps.weight"),
             gate_bias=f("ffn_gate_exps.bias"), up_bias=f("ffn_up_exps.bias"),
             down_bias=f("ffn_down_exps.bias"), router_w=f("ffn_gate_inp.weight"),
             router_b=f("ffn_gate_inp.bias"), oai_swiglu=1, norm_topk_prob=1)
    return L


@pytest.mark.parametrize("spec", [synth.GPT_OSS_MOE_LAYER, synth.TINY_GPT_OSS], ids=["gpt-oss-20b", "tiny"])
def test_router_and_moe_layer(ctx, orc, spec):
    """config 0: one GPT-OSS MoE FFN layer, one token, against the oracle's default CPU path"""
    L = _moe_layer_host(spec, seed=0)
    x = synth.moe_layer_input(spec, seed=0)
    want, want_idx, want_w = orc.moe_forward(L, x)
    H, I, E, K = spec.hidden, spec.inter, spec.experts, spec.top_k
    ones = dev(np.ones(H, np.float32))
    h0 = np.zeros(H, np.float32) + x  # the router normalises h itself; x is already RMS-normed
    d_h = dev(h0)
    xn = torch.empty(H, dtype=torch.float32, device="cuda")
    logits = torch.empty(E, dtype=torch.float32, device="cuda")
    idx = torch.empty(K, dtype=torch.int32, device="cuda")
    wts = torch.empty(K, dtype=torch.float32, device="cuda")
    # router on the already-normed input (h = None): logits from x directly, like the oracle
    xn.copy_(dev(x))
    ctx.router_topk(None, None, spec.eps, dev(L["router_w"]), dev(L["router_b"]), None, H, E, K, 0, 1,
                    xn, logits, idx, wts)
    out = torch.zeros(H, dtype=torch.float32, device="cuda")
    ctx.moe_mxfp4_decode(dev(pad_rows(L["gate"])), dev(pad_rows(L["up"])), dev(pad_rows(L["down"])),
                         dev(L["gate_bias"]), dev(L["up_bias"]), dev(L["down_bias"]), H, I, E, K, 0,
                         xn, idx, wts, out)
    ctx.sync()
    got_idx = idx.cpu().numpy()
    lg = logits.cpu().numpy()
    srt = np.sort(lg)[::-1]
    if srt[K - 1] - srt[K] > 1e-6:   # routed indices exact unless a top-k tie below 1e-6
        assert got_idx.tolist() == want_idx[0].tolist()
        np.testing.assert_allclose(wts.cpu().numpy(), want_w[0], rtol=1e-5)
        assert rel_err(out.cpu().numpy(), want[0]) < REL_TOL
    else:   # a near-tie: the layer on the GPU's own routing against the float64 restatement
        assert rel_err(out.cpu().numpy(), moe_with_routing(orc, L, x, got_idx, wts.cpu().numpy())) < REL_TOL
    del h0, d_h, ones


def test_moe_residual_accumulates(ctx, orc):
    spec = synth.TINY_GPT_OSS
    L = _moe_layer_host(spec, seed=3)
    x = synth.moe_layer_input(spec, seed=3)
    want, want_idx, want_w = orc.moe_forward(L, x)
    H, I, E, K = spec.hidden, spec.inter, spec.experts, spec.top_k
    h = np.random.default_rng(1).standard_normal(H).astype(np.float32)
    d_h = dev(h)
    ctx.moe_mxfp4_decode(dev(pad_rows(L["gate"])), dev(pad_rows(L["up"])), dev(pad_rows(L["down"])),
                         dev(L["gate_bias"]), dev(L["up_bias"]), dev(L["down_bias"]), H, I, E, K, 0,
                         dev(x), dev(want_idx[0].astype(np.int32)), dev(want_w[0]), d_h)
    ctx.sync()
    assert rel_err(d_h.cpu().numpy() - h, want[0]) < REL_TOL


def _packed(ctx, L, spec):
    """native GGUF MXFP4 stacks -> the tensor-core tile layout, through the C ABI"""
    from moe_stream_b200.engine import Context
    H, I, E = spec.hidden, spec.inter, spec.experts
    gb, db = Context.mxfp4_packed_bytes(H, I, E)
    gu = torch.empty(gb, dtype=torch.uint8, device="cuda")
    dn = torch.empty(db, dtype=torch.uint8, device="cuda")
    ctx.mxfp4_pack_experts(dev(L["gate"]), dev(L["up"]), dev(L["down"]), H, I, E, gu, dn)
    return gu, dn


@pytest.mark.parametrize("spec", [synth.GPT_OSS_MOE_LAYER, synth.TINY_GPT_OSS], ids=["gpt-oss-20b", "tiny"])
def test_moe_packed_tensor_core_layer(ctx, orc, spec):
    """config 0 on the tcgen05 block-scaled path: packed experts, x as MXFP4 residual terms"""
    L = _moe_layer_host(spec, seed=0)
    x = synth.moe_layer_input(spec, seed=0)
    want, want_idx, want_w = orc.moe_forward(L, x)
    H, I, E, K = spec.hidden, spec.inter, spec.experts, spec.top_k
    gu, dn = _packed(ctx, L, spec)
    out = torch.zeros(H, dtype=torch.float32, device="cuda")
    for _ in range(2):   # the second call checks the self-resetting split-K counters
        out.zero_()
        ctx.moe_mxfp4_decode_packed(gu, dn, dev(L["gate_bias"]), dev(L["up_bias"]), dev(L["down_bias"]), H, I, E, K,
                                    0, dev(x), dev(want_idx[0].astype(np.int32)), dev(want_w[0]), out)
        ctx.sync()
        assert rel_err(out.cpu().numpy(), want[0]) < REL_TOL
    assert ctx.error_flags() == 0


def test_moe_packed_scale_range_and_residual(ctx, orc):
    """wide e8m0 scale bytes, a residual stream to add to, and repeated experts in the routing"""
    spec = synth.TINY_GPT_OSS
    L = _moe_layer_host(spec, seed=5)
    rng = np.random.default_rng(11)
    for k in ("gate", "up", "down"):
        w = L[k].copy()
        w[::17] = rng.integers(105, 140, size=w[::17].shape, dtype=np.uint8)   # block scale bytes
        L[k] = w
    x = synth.moe_layer_input(spec, seed=5) * 7.0
    H, I, E, K = spec.hidden, spec.inter, spec.experts, spec.top_k
    idx = np.array([6, 1, 6, 3], np.int32)[:K]
    wts = np.array([0.4, 0.3, 0.2, 0.1], np.float32)[:K]
    h = rng.standard_normal(H).astype(np.float32)
    d_h = dev(h)
    gu, dn = _packed(ctx, L, spec)
    ctx.moe_mxfp4_decode_packed(gu, dn, dev(L["gate_bias"]), dev(L["up_bias"]), dev(L["down_bias"]), H, I, E, K, 0,
                                dev(x), dev(idx), dev(wts), d_h)
    # the native-layout path (already pinned against the oracle) is the reference for this routing
    ref = dev(h)
    ctx.moe_mxfp4_decode(dev(pad_rows(L["gate"])), dev(pad_rows(L["up"])), dev(pad_rows(L["down"])),
                         dev(L["gate_bias"]), dev(L["up_bias"]), dev(L["down_bias"]), H, I, E, K, 0,
                         dev(x), dev(idx), dev(wts), ref)
    ctx.sync()
    assert rel_err(d_h.cpu().numpy() - h, ref.cpu().numpy() - h) < 1e-5
    # and against the float64 restatement: the repeated expert counts once per slot (layer.rs:1415, 1822)
    assert rel_err(d_h.cpu().numpy() - h, moe_with_routing(orc, L, x, idx, wts)) < REL_TOL
    assert ctx.error_flags() == 0


PREFILL_TOL = 2e-2   # bf16 activations on the prefill path (weights exact in bf16, f32 accumulation)
PRECISE_TOL = 2e-4   # activations as bf16 hi + lo pairs (~2^-18 relative each)


@pytest.mark.parametrize("spec,n_tok", [(synth.TINY_GPT_OSS, 100), (synth.GPT_OSS_MOE_LAYER, 48)],
                         ids=["tiny-100tok", "gpt-oss-20b-48tok"])
@pytest.mark.parametrize("precise", [0, 1], ids=["bf16", "hi-lo"])
def test_moe_prefill_grouped_gemm(ctx, orc, spec, n_tok, precise):
    """config 4's MoE step: tokens sorted by expert, grouped bf16 GEMM on tcgen05, against the oracle's
    multi-token expert FFN (layer.rs:1848-1894) on the same tokens and routing"""
    L = _moe_layer_host(spec, seed=9)
    x = np.random.default_rng(9).standard_normal((n_tok, spec.hidden)).astype(np.float32)
    x /= np.sqrt((x * x).mean(-1, keepdims=True) + spec.eps)
    want, want_idx, want_w = orc.moe_forward(L, x)
    H, I, E, K = spec.hidden, spec.inter, spec.experts, spec.top_k
    gu, dn = _packed(ctx, L, spec)
    out = torch.full((n_tok, H), float("nan"), dtype=torch.float32, device="cuda")
    for _ in range(2):
        ctx.moe_mxfp4_prefill_packed(gu, dn, dev(L["gate_bias"]), dev(L["up_bias"]), dev(L["down_bias"]), H, I, E, K,
                                     0, dev(x), n_tok, dev(want_idx.astype(np.int32)), dev(want_w), out, precise)
        ctx.sync()
        got = out.cpu().numpy()
        assert np.isfinite(got).all()
        assert rel_err(got, want) < (PRECISE_TOL if precise else PREFILL_TOL)
    assert ctx.error_flags() == 0


@pytest.mark.parametrize("precise", [0, 1], ids=["bf16", "hi-lo"])
def test_moe_prefill_config4_layer_16384_tokens(ctx, orc, precise):
    """one GPT-OSS-20B MoE layer over config 4's 16,384 tokens (8 prompts x 2048): ~2048 tokens per
    expert, so every expert spans several 256-token tiles and ends in a ragged one (plus one expert
    given 300 tokens more than the rest).  The layer's output for a token depends only on that token
    and its routing, so 96 sampled tokens are checked against the oracle's multi-token layer, every
    other token for finiteness."""
    spec = synth.GPT_OSS_MOE_LAYER
    L = _moe_layer_host(spec, seed=4)
    H, I, E, K, T = spec.hidden, spec.inter, spec.experts, spec.top_k, 8 * 2048
    rng = np.random.default_rng(4)
    x = rng.standard_normal((T, H)).astype(np.float32)
    x /= np.sqrt((x * x).mean(-1, keepdims=True) + spec.eps)
    idx = np.argsort(rng.random((T, E)), axis=1)[:, :K].astype(np.int32)
    for t in range(300):   # a heavier expert 7 (no expert twice in a row)
        if 7 not in idx[t]:
            idx[t, 0] = 7
    w = rng.random((T, K)).astype(np.float32)
    w /= w.sum(1, keepdims=True)
    counts = np.bincount(idx.reshape(-1), minlength=E)
    assert counts.min() > 256 and (counts % 256 != 0).any()
    gu, dn = _packed(ctx, L, spec)
    out = torch.empty((T, H), dtype=torch.float32, device="cuda")
    ctx.moe_mxfp4_prefill_packed(gu, dn, dev(L["gate_bias"]), dev(L["up_bias"]), dev(L["down_bias"]), H, I, E, K, 0,
                                 dev(x), T, dev(idx), dev(w), out, precise)
    ctx.sync()
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    sample = np.sort(rng.choice(T, 96, replace=False))
    # reference in float64 from the oracle's dequantized experts (one expert in memory at a time)
    ref = np.zeros((len(sample), H))
    per = {"gate": I * H * 17 // 32, "up": I * H * 17 // 32, "down": H * I * 17 // 32}
    for e in range(E):
        rows = [(i, k) for i, t in enumerate(sample) for k in range(K) if idx[t, k] == e]
        if not rows:
            continue
        W = {nm: orc.dequantize(G.MXFP4, L[nm][e * per[nm]:(e + 1) * per[nm]], per[nm] * 32 // 17)
             .reshape(-1, H if nm != "down" else I).astype(np.float64) for nm in ("gate", "up", "down")}
        for i, k in rows:
            xt = x[sample[i]].astype(np.float64)
            g = W["gate"] @ xt + L["gate_bias"][e * I:(e + 1) * I]
            u = W["up"] @ xt + L["up_bias"][e * I:(e + 1) * I]
            gc = np.minimum(g, 7.0)
            a = gc / (1.0 + np.exp(-1.702 * gc)) * (np.clip(u, -7.0, 7.0) + 1.0)
            ref[i] += w[sample[i], k] * (W["down"] @ a + L["down_bias"][e * H:(e + 1) * H])
    for i, t in enumerate(sample):
        assert rel_err(got[t], ref[i]) < (PRECISE_TOL if precise else PREFILL_TOL), t
    assert ctx.error_flags() == 0


def test_router_dummy_mask_and_ties(ctx):
    H, E, K = 256, 16, 4
    w = np.zeros((E, H), np.float32)
    w[:, 0] = np.arange(E, dtype=np.float32)       # logit e = e * x0
    w[15] = 0.5                                      # constant row -> treated as dummy by the loader
    x = np.zeros(H, np.float32); x[0] = 1.0
    mask = np.zeros(E, np.uint8); mask[14] = 1
    w[13, 0] = 12.0                                  # tie 12 == 12: lower index (12) first
    xn = dev(x); logits = torch.empty(E, device="cuda"); idx = torch.empty(K, dtype=torch.int32, device="cuda")
    wts = torch.empty(K, device="cuda")
    ctx.router_topk(None, None, 1e-5, dev(w), None, dev(mask), H, E, K, 0, 1, xn, logits, idx, wts)
    ctx.sync()
    # logits: e for e <= 12, 12 for e = 13, -inf for the masked 14, 0.5 for 15
    assert idx.cpu().tolist() == [12, 13, 11, 10]


# ---------------- whole model ----------------
@pytest.fixture(scope="module")
def tiny_path(tmp_path_factory):
    d = tmp_path_factory.mktemp("tiny")
    p = str(d / "tiny_gpt_oss.gguf")
    synth.write_model(p, synth.TINY_GPT_OSS, seed=7)
    return p


def test_tiny_model_greedy_tokens_match_golden(ctx, tiny_path):
    from moe_stream_b200.engine import Engine
    f = np.load(os.path.join(GOLD, "tiny_models.npz"))
    eng = Engine.open(tiny_path, max_seq_len=256, ctx=ctx)
    toks = eng.generate(f["tiny_gpt_oss_prompt"], 16)
    assert toks == f["tiny_gpt_oss_tokens"].tolist()
    eng.close()


def test_tiny_model_logits_and_hidden(ctx, orc, tiny_path):
    from moe_stream_b200.engine import Engine
    f = np.load(os.path.join(GOLD, "tiny_models.npz"))
    prompt = f["tiny_gpt_oss_prompt"]
    eng = Engine.open(tiny_path, max_seq_len=256, ctx=ctx)
    logits = eng.forward(prompt)
    assert rel_err(logits, f["tiny_gpt_oss_logits"]) < REL_TOL
    assert rel_err(eng.last_hidden(), f["tiny_gpt_oss_hidden"]) < REL_TOL
    # routed experts of the last position, every layer, against the oracle
    om = orc.Model(tiny_path, max_seq_len=256)
    om.forward(prompt)
    import ctypes as C
    k, nl = synth.TINY_GPT_OSS.top_k, synth.TINY_GPT_OSS.layers
    oi = np.empty(nl * k, np.int32); ow = np.empty(nl * k, np.float32)
    orc.lib().orc_model_last_routing(om.h, oi.ctypes.data_as(C.POINTER(C.c_int32)), ow.ctypes.data_as(C.POINTER(C.c_float)))
    for layer in range(nl):
        gi, gw = eng.last_routing(layer)
        assert gi.tolist() == oi[layer * k:(layer + 1) * k].tolist()
        np.testing.assert_allclose(gw, ow[layer * k:(layer + 1) * k], rtol=1e-4)
    om.close()
    eng.close()


def test_graph_and_stream_paths_agree(ctx, tiny_path):
    from moe_stream_b200.engine import Engine
    f = np.load(os.path.join(GOLD, "tiny_models.npz"))
    eng = Engine.open(tiny_path, max_seq_len=256, ctx=ctx)
    eng.set_graph(False)
    a = eng.generate(f["tiny_gpt_oss_prompt"], 8)
    eng.set_graph(True)
    b = eng.generate(f["tiny_gpt_oss_prompt"], 8)
    assert a == b == f["tiny_gpt_oss_tokens"][:8].tolist()
    # decode_step with host buffers gives the same continuation
    eng.clear_cache()
    eng.forward(f["tiny_gpt_oss_prompt"][:-1])
    nxt = eng.decode_step(int(f["tiny_gpt_oss_prompt"][-1]))
    assert nxt == b[0]
    eng.close()


def test_in_memory_upload_matches_file(ctx, tiny_path):
    from moe_stream_b200.engine import Engine
    f = np.load(os.path.join(GOLD, "tiny_models.npz"))
    m = synth.build_model(synth.TINY_GPT_OSS, seed=7)
    eng = Engine.from_model(m, max_seq_len=256, ctx=ctx)
    assert eng.generate(f["tiny_gpt_oss_prompt"], 16) == f["tiny_gpt_oss_tokens"].tolist()
    eng.close()


@pytest.fixture(scope="module")
def tiny_qwen_path(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("tq") / "tiny_qwen3.gguf")
    synth.write_model(p, synth.TINY_QWEN3, seed=7)
    return p


def test_tiny_model_native_expert_path(ctx, tiny_path, monkeypatch):
    """MS_MOE_TC=0 keeps the native-block mma.sync expert kernels; same golden tokens"""
    from moe_stream_b200.engine import Engine
    monkeypatch.setenv("MS_MOE_TC", "0")
    f = np.load(os.path.join(GOLD, "tiny_models.npz"))
    eng = Engine.open(tiny_path, max_seq_len=256, ctx=ctx)
    assert eng.generate(f["tiny_gpt_oss_prompt"], 16) == f["tiny_gpt_oss_tokens"].tolist()
    eng.close()


def test_tiny_qwen3_q4k_q6k_model(ctx, orc, tiny_qwen_path):
    """Qwen3-shaped model: Q4_K gate/up, Q6_K down, QK-norm, softmax over all experts + renorm"""
    from moe_stream_b200.engine import Engine
    f = np.load(os.path.join(GOLD, "tiny_models.npz"))
    prompt = f["tiny_qwen3_prompt"]
    eng = Engine.open(tiny_qwen_path, max_seq_len=256, ctx=ctx)
    assert eng.generate(prompt, 16) == f["tiny_qwen3_tokens"].tolist()
    eng.clear_cache()
    assert rel_err(eng.forward(prompt), f["tiny_qwen3_logits"]) < REL_TOL
    assert rel_err(eng.last_hidden(), f["tiny_qwen3_hidden"]) < REL_TOL
    eng.close()


def test_long_context_sliding_window(ctx, orc, tmp_path):
    """positions past the 8-slot sliding window ring, full layers over 200+ positions"""
    from moe_stream_b200.engine import Engine
    p = str(tmp_path / "t.gguf")
    synth.write_model(p, synth.TINY_GPT_OSS, seed=9)
    prompt = synth.prompt_ids(synth.TINY_GPT_OSS, 150, seed=9)
    eng = Engine.open(p, max_seq_len=512, ctx=ctx)
    om = orc.Model(p, max_seq_len=512)
    got = eng.generate(prompt, 40)
    want = om.generate(prompt, 40).tolist()
    assert got == want
    om.close()
    eng.close()


# ---- hybrid blocks: Gated DeltaNet decode (deltanet.rs:204-543), shared expert (layer.rs:2250-2293) ----


def _dn_device(d):
    out = dict(d)
    for k in ("qkv", "gate", "ba", "out"):
        out[k] = dev(pad_rows(d[k]))
    for k in ("conv1d", "ssm_a", "dt_bias", "norm"):
        out[k] = dev(d[k])
    return out


@pytest.mark.parametrize("shape,qtype", [
    (dict(), G.F32),
    (dict(nk=1, hkd=32, nv=2, ks=3), G.F32),
    (dict(hidden=2048, nk=16, hkd=128, nv=32, ks=4), G.Q4_K),     # Qwen3-Next linear-attention layer
    (dict(hidden=512, nk=4, hkd=128, nv=8, ks=4), G.Q6_K),
])
def test_deltanet_decode_multi_step(ctx, orc, shape, qtype):
    d = hs.deltanet_layer(11, qtype=qtype, **shape)
    dd = _dn_device(d)
    nv, hkd, hvd, ks = d["n_v_heads"], d["head_k_dim"], d["head_v_dim"], d["conv_kernel"]
    conv_dim = 2 * d["n_k_heads"] * hkd + nv * hvd
    cs = np.zeros((conv_dim, ks - 1), np.float32)
    rs = np.zeros((nv, hkd, hvd), np.float32)
    cs_d, rs_d = dev(cs), dev(rs)
    y_d = torch.empty(d["hidden"], dtype=torch.float32, device="cuda")
    rng = np.random.default_rng(3)
    for step in range(6):
        x = rng.standard_normal(d["hidden"]).astype(np.float32)
        want = orc.deltanet_step(d, x, cs, rs)
        ctx.deltanet_decode(dd, dev(x), cs_d, rs_d, y_d)
        ctx.sync()
        assert rel_err(y_d.cpu().numpy(), want) < REL_TOL, step
        assert rel_err(rs_d.cpu().numpy(), rs) < REL_TOL, step
        assert rel_err(cs_d.cpu().numpy(), cs) < REL_TOL, step


def test_deltanet_decode_rejects_unsupported_head_dim(ctx):
    from moe_stream_b200._lib import MsError
    d = _dn_device(hs.deltanet_layer(1, hvd=64))
    with pytest.raises(MsError):
        ctx.deltanet_decode(d, torch.zeros(d["hidden"], device="cuda"),
                            torch.zeros(4096, device="cuda"), torch.zeros(1 << 16, device="cuda"),
                            torch.zeros(d["hidden"], device="cuda"))


@pytest.mark.parametrize("hidden,inter,gu_q,down_q,gated", [
    (256, 128, G.F32, G.F32, True),
    (2048, 512, G.Q4_K, G.Q6_K, True),      # Qwen3-Next shared expert shape
    (512, 256, G.Q4_K, G.Q4_K, False),
])
def test_shared_expert(ctx, orc, hidden, inter, gu_q, down_q, gated):
    e = hs.shared_expert(9, hidden, inter, gu_q, down_q, gated)
    rng = np.random.default_rng(hidden + inter)
    x = rng.standard_normal(hidden).astype(np.float32)
    y0 = rng.standard_normal(hidden).astype(np.float32)
    want = orc.shared_expert(e["gu_q"], e["gate"], e["up"], e["down_q"], e["down"], e["gate_inp"], hidden, inter,
                             x, y0.copy())
    y = dev(y0)
    gi = dev(e["gate_inp"]) if gated else None
    ctx.shared_expert(gu_q, dev(pad_rows(e["gate"])), dev(pad_rows(e["up"])), down_q, dev(pad_rows(e["down"])), gi,
                      hidden, inter, dev(x), y)
    ctx.sync()
    assert rel_err(y.cpu().numpy(), want) < REL_TOL


# ---- lockstep batch decode (Engine::forward over input_ids [B, T], engine.rs:1869-2006) ----


def _batch_prompts(spec, B, T, seed):
    return np.stack([synth.prompt_ids(spec, T, seed=seed + b) for b in range(B)])


def test_batch_decode_qwen3_matches_oracle_per_sequence(ctx, orc, tiny_qwen_path):
    """B = 5 sequences (not a multiple of the 4-token MMA groups): each one's greedy tokens equal
    the oracle's single-sequence generation; last-position logits match the bs1 engine"""
    from moe_stream_b200.engine import Engine
    B, T, N = 5, 12, 10
    prompts = _batch_prompts(synth.TINY_QWEN3, B, T, 40)
    eng = Engine.open(tiny_qwen_path, max_seq_len=128, ctx=ctx)
    eng.batch_open(B)
    got = eng.batch_generate(prompts, N)
    om = orc.Model(tiny_qwen_path, max_seq_len=128)
    for b in range(B):
        om.clear_cache()
        assert got[b].tolist() == om.generate(prompts[b], N).tolist(), b
    om.close()
    eng.batch_clear()
    eng.batch_forward(prompts)
    bl = eng.batch_last_logits()
    for b in (0, B - 1):
        eng.clear_cache()
        assert rel_err(bl[b], eng.forward(prompts[b])) < REL_TOL
    eng.close()


def test_batch_decode_gpt_oss_native_mxfp4_sliding_window(ctx, orc, tmp_path, monkeypatch):
    """native-layout MXFP4 experts with biases and OAI SwiGLU, sinks, 8-slot SWA ring passed"""
    from moe_stream_b200.engine import Engine
    monkeypatch.setenv("MS_MOE_TC", "0")
    p = str(tmp_path / "g.gguf")
    synth.write_model(p, synth.TINY_GPT_OSS, seed=5)
    B, T, N = 3, 20, 12
    prompts = _batch_prompts(synth.TINY_GPT_OSS, B, T, 70)
    eng = Engine.open(p, max_seq_len=128, ctx=ctx)
    eng.batch_open(B)
    got = eng.batch_generate(prompts, N)
    om = orc.Model(p, max_seq_len=128)
    for b in range(B):
        om.clear_cache()
        assert got[b].tolist() == om.generate(prompts[b], N).tolist(), b
    om.close()
    eng.close()


def test_batch_decode_full_batch_matches_single_sequence_engine(ctx, tiny_qwen_path):
    """B = 32 (the maximum): every sequence equals the bs1 engine's generation"""
    from moe_stream_b200.engine import Engine
    B, T, N = 32, 6, 6
    prompts = _batch_prompts(synth.TINY_QWEN3, B, T, 100)
    eng = Engine.open(tiny_qwen_path, max_seq_len=64, ctx=ctx)
    eng.batch_open(B)
    got = eng.batch_generate(prompts, N)
    for b in range(B):
        assert got[b].tolist() == eng.generate(prompts[b], N), b
    # exact numerics: QKV, attention, O, router, 2 expert kernels, residual per layer; LM head + refine
    assert eng.batch_kernels_per_step == 2 + 7 * eng.config.layers + 4
    eng.close()


def test_batch_open_rejects_packed_experts(ctx, tiny_path):
    from moe_stream_b200._lib import MsError
    from moe_stream_b200.engine import Engine
    eng = Engine.open(tiny_path, max_seq_len=64, ctx=ctx)
    with pytest.raises(MsError):
        eng.batch_open(4)
    eng.close()


@pytest.mark.parametrize("head_dim", [64, 128])
def test_batch_decode_gqa8_attention(ctx, orc, tmp_path, head_dim):
    """8 query heads per kv head over 62 positions (several 32-position attention chunks), batched
    and single-sequence, against the oracle's last-position logits.

    Every position re-quantizes each projection input to Q8_0 (candle QMatMul numerics); with
    q_dim 2048 a different f32 summation order moves about one activation code per position by one
    step, so the logits carry 1e-3 to 5e-3 of rounding noise relative to the oracle (the batched
    and single-sequence GPU paths agree to ~1e-7 until such a flip).  The bound below is 1e-2, and
    the greedy token is compared wherever the oracle's top-2 margin exceeds that noise."""
    from dataclasses import replace
    from moe_stream_b200.engine import Engine
    spec = replace(synth.TINY_QWEN3, name="tiny-qwen3-gqa8", heads=16, kv_heads=2, head_dim=head_dim)
    p = str(tmp_path / "q.gguf")
    synth.write_model(p, spec, seed=13)
    B, T = 3, 62
    prompts = _batch_prompts(spec, B, T, 200)
    eng = Engine.open(p, max_seq_len=128, ctx=ctx)
    eng.batch_open(B)
    eng.batch_forward(prompts)
    bl = eng.batch_last_logits()
    om = orc.Model(p, max_seq_len=128)
    for b in range(B):
        om.clear_cache()
        want = om.forward(prompts[b])
        eng.clear_cache()
        single = eng.forward(prompts[b])
        scale = np.abs(want).max()
        assert rel_err(bl[b], want) < 1e-2 and rel_err(single, want) < 1e-2, b
        top2 = np.sort(want)[-2:]
        if (top2[1] - top2[0]) / scale > 2e-2:
            assert int(bl[b].argmax()) == int(want.argmax()) == int(single.argmax()), b
    om.close()
    eng.close()


# ---- the per-dispatch seam: RoPE (fused_rope_metal) and one attention half-layer ----


@pytest.mark.parametrize("heads,hd,rot,n_tok", [(64, 64, 64, 1), (8, 128, 128, 5), (16, 256, 64, 3)])
def test_rope_bit_exact(ctx, orc, heads, hd, rot, n_tok):
    """NeoX rotation of the first rot dims (partial rotary passes the rest through), bit for bit"""
    rng = np.random.default_rng(heads + hd + rot)
    cs, sn = orc.rope_tables(rot, 4096, 150000.0)
    pos = rng.integers(0, 4096, n_tok)
    x = rng.standard_normal((n_tok, heads, hd)).astype(np.float32) * 3
    y = torch.empty(x.size, dtype=torch.float32, device="cuda")
    ctx.rope(dev(x), dev(cs[pos]), dev(sn[pos]), n_tok, heads, hd, rot, y)
    ctx.sync()
    want = orc.rope(x, cs[pos], sn[pos], n_tok, heads, hd, rot)
    assert np.array_equal(y.cpu().numpy().view(np.uint32), want.reshape(-1).view(np.uint32))


def _attn_layer(seed, H, nh, nkv, hd, rot, window=0, sinks=False, bias=False, qk_norm=False, theta=150000.0,
                q_gate=False):
    rng = np.random.default_rng(seed)
    Dq, Dkv = nh * hd, nkv * hd
    Dqw = 2 * Dq if q_gate else Dq   # hybrid models: [Q_h, gate_h] per head in the Q projection
    d = dict(hidden=H, heads=nh, kv_heads=nkv, head_dim=hd, rot_dim=rot, eps=1e-5, rope_theta=theta, window=window,
             attn_norm=(1 + 0.1 * rng.standard_normal(H)).astype(np.float32),
             wq=synth.rand_q8_0(rng, Dqw * H), wk=synth.rand_q8_0(rng, Dkv * H), wv=synth.rand_q8_0(rng, Dkv * H),
             wo=synth.rand_q8_0(rng, H * Dq), q_gate=int(q_gate))
    if bias:
        for k, n in (("bq", Dqw), ("bk", Dkv), ("bv", Dkv), ("bo", H)):
            d[k] = (rng.standard_normal(n) * 0.01).astype(np.float32)
    if sinks:
        d["sinks"] = rng.standard_normal(nh).astype(np.float32)
    if qk_norm:
        d["q_norm"] = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
        d["k_norm"] = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    return d


@pytest.mark.parametrize("shape", [
    dict(H=2880, nh=64, nkv=8, hd=64, rot=64, window=128, sinks=True, bias=True, steps=150),    # GPT-OSS SWA layer
    dict(H=2880, nh=64, nkv=8, hd=64, rot=64, sinks=True, bias=True, steps=40),                 # GPT-OSS full layer
    dict(H=2048, nh=32, nkv=4, hd=128, rot=128, qk_norm=True, theta=1e6, steps=40),            # Qwen3-30B-A3B
    dict(H=2048, nh=16, nkv=2, hd=256, rot=64, qk_norm=True, theta=1e7, steps=24),             # head_dim 256, rotary 0.25
    dict(H=2048, nh=16, nkv=2, hd=256, rot=64, qk_norm=True, theta=1e7, q_gate=True, steps=24),  # hybrid: gated Q
    dict(H=1024, nh=16, nkv=2, hd=64, rot=16, qk_norm=True, bias=True, q_gate=True, steps=40),   # gated, exact kernel
], ids=["gpt-oss-swa", "gpt-oss-full", "qwen3", "hd256-partial-rope", "hybrid-gated-hd256", "gated-hd64"])
def test_attn_layer_decode(ctx, orc, shape):
    """ms_attn_layer_decode step by step against the oracle's attention half-layer (fresh input each
    step; both keep their own K/V).  Head dims 32/64/128 run the order-independent kernel: every
    reduction in double, rounded once, so the QKV input's Q8_0 codes, q/k/v, the softmax, the
    attention output and its Q8_0 codes, and the O projection all come out bit-identical to the
    oracle's -- the residual stream after every step must match exactly.  Head dim 256 runs the
    split-K f32 kernel (within 1e-3)."""
    shape = dict(shape)
    steps = shape.pop("steps")
    theta = shape.pop("theta", 150000.0)
    d = _attn_layer(17, theta=theta, **shape)
    H, nkv, hd, window = d["hidden"], d["kv_heads"], d["head_dim"], d["window"]
    cap = window if window else steps
    cs, sn = orc.rope_tables(d["rot_dim"], steps, theta)
    ostate = orc.AttnState(d)
    wqkv = np.concatenate([d["wq"], d["wk"], d["wv"]])
    bqkv = np.concatenate([d["bq"], d["bk"], d["bv"]]) if "bq" in d else None
    kc = torch.zeros(nkv * cap * hd, device="cuda")
    vc = torch.zeros_like(kc)
    g = dict(hidden=H, heads=d["heads"], kv_heads=nkv, head_dim=hd, rot_dim=d["rot_dim"], eps=d["eps"], window=window,
             cap=cap, attn_norm=dev(d["attn_norm"]), wqkv=dev(pad_rows(wqkv)), wo=dev(pad_rows(d["wo"])),
             bqkv=dev(bqkv) if bqkv is not None else None, bo=dev(d["bo"]) if "bo" in d else None,
             sinks=dev(d["sinks"]) if "sinks" in d else None, q_norm=dev(d["q_norm"]) if "q_norm" in d else None,
             k_norm=dev(d["k_norm"]) if "k_norm" in d else None, k_cache=kc, v_cache=vc, cos_t=dev(cs), sin_t=dev(sn),
             q_gate=d["q_gate"])
    rng = np.random.default_rng(5)
    exact = hd <= 128
    for pos in range(steps):
        h = rng.standard_normal(H).astype(np.float32)
        want = ostate.step(h)
        hd_ = dev(h)
        ctx.attn_layer_decode(g, pos, hd_)
        ctx.sync()
        got = hd_.cpu().numpy()
        if exact:
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
                f"position {pos}: {int((got != want).sum())} elements differ, max {rel_err(got - h, want - h):.3g}"
        else:
            assert rel_err(got - h, want - h) < REL_TOL, f"position {pos}"
    assert ctx.error_flags() == 0


# ---- multi-token forward (prompt prefill) through the model, against the oracle's ----


def _prefill_vs_oracle(ctx, orc, path, spec, prompt, mode, tol, n_gen=12):
    from moe_stream_b200.engine import Engine
    eng = Engine.open(path, max_seq_len=len(prompt) + 64, ctx=ctx)
    eng.set_prefill(mode)
    eng.set_trace(True)
    om = orc.Model(path, max_seq_len=len(prompt) + 64)
    logits = eng.forward(prompt)
    want = om.forward(prompt)
    assert rel_err(logits, want) < tol
    assert rel_err(eng.last_hidden(), om.last_hidden()) < tol
    hid, lg = eng.layer_trace()
    ohid, olg = om.layer_trace(spec.layers, spec.experts)
    for layer in range(spec.layers):
        assert rel_err(hid[layer], ohid[layer]) < tol, layer
    oi, _ = om.last_routing(spec.layers, spec.top_k)
    for layer in range(spec.layers):
        srt = np.sort(olg[layer])[::-1]
        if srt[spec.top_k - 1] - srt[spec.top_k] > 1e-6:
            assert eng.last_routing(layer)[0].tolist() == oi[layer].tolist(), layer
    if n_gen:
        # greedy continuation after the batched prompt equals the oracle's generation
        got = eng.generate(prompt, n_gen)
        om.clear_cache()
        assert got == om.generate(prompt, n_gen).tolist()
    om.close()
    eng.close()


@pytest.mark.parametrize("n_prompt", [40, 97])
def test_prefill_gpt_oss_tiny_sliding_window(ctx, orc, tiny_path, n_prompt):
    """batched prompt (longer than the 8-slot window, so the chunk reads its own keys past the ring),
    sinks, biases, MXFP4 experts on the hi/lo grouped GEMM: logits, every layer's residual stream and
    routing within 1e-3 of the oracle's multi-token forward, then identical greedy tokens"""
    prompt = synth.prompt_ids(synth.TINY_GPT_OSS, n_prompt, seed=31)
    _prefill_vs_oracle(ctx, orc, tiny_path, synth.TINY_GPT_OSS, prompt, 1, REL_TOL)


def test_prefill_gpt_oss_tiny_bf16_mode(ctx, orc, tiny_path):
    """mode 2 (plain bf16 expert activations) within the north star's 2e-2 prefill bound"""
    prompt = synth.prompt_ids(synth.TINY_GPT_OSS, 64, seed=32)
    _prefill_vs_oracle(ctx, orc, tiny_path, synth.TINY_GPT_OSS, prompt, 2, PREFILL_TOL, n_gen=0)


def test_prefill_qwen3_tiny_kquant(ctx, orc, tiny_qwen_path):
    """QK-norm, K-quant experts grouped 32 tokens at a time, renormalised routing.  The batched
    prompt path is not order-independent (f32 online-softmax attention, f16 hi/lo expert MMAs), so a
    Q8_0 activation code can round the other way; it is held to the north star's prefill bound
    (2e-2), and the greedy continuation must still equal the oracle's."""
    prompt = synth.prompt_ids(synth.TINY_QWEN3, 70, seed=33)
    _prefill_vs_oracle(ctx, orc, tiny_qwen_path, synth.TINY_QWEN3, prompt, 1, PREFILL_TOL)


def test_prefill_longer_than_one_chunk(ctx, orc, tiny_path):
    """2100 prompt tokens: two batched passes (2048 + 52), the second attending over the first's
    cache, against the oracle's single multi-token forward"""
    prompt = synth.prompt_ids(synth.TINY_GPT_OSS, 2100, seed=34)
    _prefill_vs_oracle(ctx, orc, tiny_path, synth.TINY_GPT_OSS, prompt, 1, REL_TOL, n_gen=4)


def test_prefill_then_decode_matches_stepwise(ctx, tiny_qwen_path):
    """the batched prompt leaves the same cache and state as one decode step per token"""
    from moe_stream_b200.engine import Engine
    prompt = synth.prompt_ids(synth.TINY_QWEN3, 33, seed=35)
    eng = Engine.open(tiny_qwen_path, max_seq_len=128, ctx=ctx)
    eng.set_prefill(0)
    a = eng.generate(prompt, 10)
    la = eng.token_log()
    eng.set_prefill(1)
    b = eng.generate(prompt, 10)
    assert a == b and eng.token_log() == la and eng.seq_len == len(prompt) + 9
    eng.close()


# ---- sampling (SamplingParams::sample, engine.rs:124-208) ----
def _sample_cases(V, n, seed):
    rng = np.random.default_rng(seed)
    for t in range(n):
        lg = (rng.standard_normal(V) * [1.0, 3.0, 8.0][t % 3]).astype(np.float32)
        if t % 4 == 1:
            lg[rng.integers(0, V, 8)] = lg.max()                      # ties at the maximum
        if t % 4 == 2:
            lg[: V // 2] = np.float32(0.5)                             # ties inside the nucleus boundary
        counts = rng.integers(0, 3, V).astype(np.uint32) if t % 3 == 0 else None
        T = [0.0, 1.0, 0.7, 1.3][t % 4]
        top_p = [1.0, 0.9, 0.5, 0.02, 0.999][t % 5]
        pen = [1.0, 1.2][t % 2]
        yield lg, counts, T, top_p, pen, float(rng.random())


@pytest.mark.parametrize("V,n", [(50, 40), (3000, 40), (201088, 12)])
def test_sample_matches_oracle(ctx, orc, V, n):
    """ms_sample picks the oracle's token: penalty, greedy ties (last maximum), temperature, the
    top-p nucleus with ties at its boundary in index order, the draw"""
    work = torch.empty(V, dtype=torch.float32, device="cuda")
    tok = torch.empty(1, dtype=torch.int32, device="cuda")
    for i, (lg, counts, T, top_p, pen, r) in enumerate(_sample_cases(V, n, V)):
        ctx.sample(dev(lg), dev(counts) if counts is not None else None, T, top_p, pen, r, work, tok)
        torch.cuda.synchronize()
        want = orc.sample(lg, counts, T, top_p, pen, r)
        assert int(tok.item()) == want, (i, T, top_p, pen, r)
    assert ctx.error_flags() == 0


def test_model_sampled_generation(ctx, tiny_path):
    """generate_sampled on the device: temperature 0 gives the greedy sequence, a seed reproduces its
    sequence and another seed changes it, and the prompt positions draw nothing (the first draw
    follows the last prompt token)"""
    from moe_stream_b200.engine import Engine
    f = np.load(os.path.join(GOLD, "tiny_models.npz"))
    prompt = f["tiny_gpt_oss_prompt"]
    eng = Engine.open(tiny_path, max_seq_len=256, ctx=ctx)
    try:
        greedy = eng.generate(prompt, 12)
        assert eng.generate_sampled(prompt, 12, temperature=0.0) == greedy
        a = eng.generate_sampled(prompt, 12, temperature=1.0, top_p=0.9, repetition_penalty=1.1, seed=5)
        b = eng.generate_sampled(prompt, 12, temperature=1.0, top_p=0.9, repetition_penalty=1.1, seed=5)
        c = eng.generate_sampled(prompt, 12, temperature=1.0, top_p=0.9, repetition_penalty=1.1, seed=6)
        assert a == b and a != c
        V = eng.config.vocab
        assert all(0 <= t < V for t in a)
        assert ctx.error_flags() == 0
    finally:
        eng.close()
