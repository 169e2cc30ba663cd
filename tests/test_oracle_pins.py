"""Pins of the CPU oracle: the reference's own unit-test values, an independent
GGML dequantizer (golden fixtures), and algorithm-level properties."""
import os

import numpy as np
import pytest

from moe_stream_b200 import gguf as G
from moe_stream_b200 import synth

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def bits_equal(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    both_nan = np.isnan(a) & np.isnan(b)
    return bool(np.all((a.view(np.uint32) == b.view(np.uint32)) | both_nan))


# ---- reference unit tests (values quoted from the reference's #[cfg(test)] blocks) ----
def test_fp16_known_answers(orc):  # gguf/dequant.rs:809-816
    L = orc.lib()
    assert L.orc_fp16_to_f32(0x3C00) == 1.0
    assert L.orc_fp16_to_f32(0x0000) == 0.0
    assert L.orc_fp16_to_f32(0xBC00) == -1.0


def test_q4k_single_block(orc):  # gguf/dequant.rs:819-837
    b = np.zeros(144, np.uint8)
    b[1] = 0x3C
    b[4:8] = 1
    out = orc.dequantize(G.Q4_K, b, 256)
    assert out.size == 256 and out[0] == 0.0


def test_q6k_zero_block(orc):  # gguf/dequant.rs:840-844
    out = orc.dequantize(G.Q6_K, np.zeros(210, np.uint8), 256)
    assert out.size == 256 and np.all(out == 0)


def test_rms_norm_basic(orc):  # ops/norm.rs:45-56
    y = orc.rms_norm(np.array([[1, 2, 3, 4]], np.float32), np.ones(4, np.float32), 1e-6)
    assert abs(y[0, 0] - 0.3651) < 0.01 and abs(y[0, 3] - 1.4606) < 0.01


def test_silu_and_mul(orc):  # ops/activation.rs:68-78
    y = orc.silu_and_mul(np.array([1, -1, 2, 0], np.float32), np.ones(4, np.float32))
    assert abs(y[0] - 0.7311) < 0.01 and abs(y[1] + 0.2689) < 0.01 and abs(y[3]) < 0.001


def test_rope_tables(orc):  # ops/attention.rs:288-300
    c, s = orc.rope_tables(128, 32, 10000.0)
    assert c.shape == (32, 64) and s.shape == (32, 64)
    assert abs(c[0, 0] - 1.0) < 1e-5 and abs(s[0, 0]) < 1e-5


def test_sdpa_single_token(orc):  # ops/attention.rs:302-328
    import ctypes as C
    q = np.array([1, 0, 0, 0, 0, 1, 0, 0], np.float32)
    v = np.arange(1, 9, dtype=np.float32)
    out = np.empty(8, np.float32)
    fp = C.POINTER(C.c_float)
    orc.lib().orc_sdpa.argtypes = [fp, fp, fp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_double,
                                   C.c_int, fp, C.c_int, fp]
    orc.lib().orc_sdpa(q.ctypes.data_as(fp), q.ctypes.data_as(fp), v.ctypes.data_as(fp), 2, 2, 1, 1, 4,
                       0.5, 0, fp(), 0, out.ctypes.data_as(fp))
    assert abs(out[0] - 1.0) < 1e-5 and abs(out[4] - 5.0) < 1e-5


def test_oai_swiglu_clamp(orc):  # model/train.rs:1152-1186
    y = orc.swiglu_oai(np.array([1, -1, 5, 10], np.float32), np.array([0.5, -0.5, 2, 3], np.float32))
    assert abs(y[3] - 28.0) < 0.5


# ---- independent GGML dequantizer (gguf 0.19.0) via committed fixtures ----
@pytest.mark.parametrize("key,qtype", [("mxfp4", G.MXFP4), ("q4_k", G.Q4_K), ("q6_k", G.Q6_K),
                                       ("q8_0", G.Q8_0), ("f16", G.F16)])
def test_dequant_matches_golden(orc, key, qtype):
    f = np.load(os.path.join(GOLD, "dequant_kat.npz"))
    raw, want = f[f"{key}_raw"], f[f"{key}_out"]
    got = orc.dequantize(qtype, raw, want.size)
    assert bits_equal(got, want)


def test_e8m0_edges(orc):  # dequant.rs:589-597
    L = orc.lib()
    assert L.orc_e8m0_to_f32_half(0) == 2.0 ** -128
    assert L.orc_e8m0_to_f32_half(1) == 2.0 ** -127
    assert L.orc_e8m0_to_f32_half(2) == 2.0 ** -126
    assert L.orc_e8m0_to_f32_half(128) == 1.0
    assert L.orc_e8m0_to_f32_half(255) == 2.0 ** 127


def test_mxfp4_nibble_layout(orc):  # low nibble -> j, high nibble -> j+16
    b = np.zeros(17, np.uint8)
    b[0] = 128
    b[1] = 0x71        # element 0 = LUT[1] = 1, element 16 = LUT[7] = 12
    b[16] = 0x8F       # element 15 = LUT[15] = -12, element 31 = LUT[8] = -0
    y = orc.dequantize(G.MXFP4, b, 32)
    assert y[0] == 1.0 and y[16] == 12.0 and y[15] == -12.0
    assert y[31] == 0.0 and np.signbit(y[31])


# ---- algorithm properties ----
def test_topk_ties_lower_index_first(orc):  # stable sort, layer.rs:2358
    logits = np.array([[1.0, 3.0, 3.0, 2.0, 3.0]], np.float32)
    idx, w = orc.top_k_routing(logits, 3, True, True)
    assert idx.tolist() == [[1, 2, 4]]
    assert np.allclose(w, 1 / 3)
    idx, w = orc.top_k_routing(logits, 2, True, False)
    assert idx.tolist() == [[1, 2]] and np.allclose(w.sum(), 1.0)


def test_topk_softmax_modes(orc):
    rng = np.random.default_rng(0)
    lg = rng.standard_normal((5, 32)).astype(np.float32)
    idx, w = orc.top_k_routing(lg, 4, False, True)   # GPT-OSS: softmax over selected
    for t in range(5):
        sel = np.argsort(-lg[t], kind="stable")[:4]
        assert idx[t].tolist() == sel.tolist()
        e = np.exp(lg[t, sel] - lg[t, sel].max())
        np.testing.assert_allclose(w[t], e / e.sum(), rtol=1e-6)
    idx, w = orc.top_k_routing(lg, 4, False, False)  # softmax over all, no renorm
    for t in range(5):
        p = np.exp(lg[t] - lg[t].max()); p /= p.sum()
        np.testing.assert_allclose(w[t], p[idx[t]], rtol=1e-5)


def test_mxfp4_matvec_vs_dequant_gemv(orc):
    rng = np.random.default_rng(3)
    rows, cols = 64, 256
    w = synth.rand_mxfp4(rng, rows * cols)
    x = rng.standard_normal(cols).astype(np.float32)
    a = orc.mxfp4_matvec_mul(w, x, rows, cols)
    b = orc.gemv(G.MXFP4, w, rows, cols, x)
    dense = orc.dequantize(G.MXFP4, w, rows * cols).reshape(rows, cols).astype(np.float64)
    ref = dense @ x.astype(np.float64)
    np.testing.assert_allclose(a, ref, rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(b, ref, rtol=1e-4, atol=1e-6)


def test_q8_0_activation_quant_vs_exact(orc):
    rng = np.random.default_rng(4)
    rows, cols = 32, 512
    w = synth.rand_q8_0(rng, rows * cols)
    x = rng.standard_normal(cols).astype(np.float32)
    exact = orc.q8_0_gemv(w, rows, cols, x, mode=0)
    actq = orc.q8_0_gemv(w, rows, cols, x, mode=1)
    dense = orc.dequantize(G.Q8_0, w, rows * cols).reshape(rows, cols).astype(np.float64)
    np.testing.assert_allclose(exact, dense @ x, rtol=1e-4, atol=1e-5)
    # the activation-quantization gap candle's QMatMul introduces (~1e-2 relative, not a bug)
    rel = np.abs(actq - exact).max() / np.abs(exact).max()
    assert rel < 5e-2


def test_quantize_q8_0_matches_numpy_synth(orc):
    rng = np.random.default_rng(5)
    x = rng.standard_normal(32 * 40).astype(np.float32) * 0.02
    assert np.array_equal(orc.quantize_q8_0(x), synth.quantize_q8_0(x))


def test_tiny_model_regression(orc, tmp_path):
    f = np.load(os.path.join(GOLD, "tiny_models.npz"))
    for name, spec in (("tiny_gpt_oss", synth.TINY_GPT_OSS), ("tiny_qwen3", synth.TINY_QWEN3)):
        p = str(tmp_path / f"{name}.gguf")
        synth.write_model(p, spec, seed=7)
        m = orc.Model(p, max_seq_len=256)
        toks = m.generate(f[f"{name}_prompt"], 16)
        assert toks.tolist() == f[f"{name}_tokens"].tolist()
        m.clear_cache()
        np.testing.assert_allclose(m.forward(f[f"{name}_prompt"]), f[f"{name}_logits"], rtol=1e-5, atol=1e-6)
        m.close()


def test_gguf_roundtrip(tmp_path):
    m = synth.build_model(synth.TINY_GPT_OSS, seed=1)
    p = str(tmp_path / "t.gguf")
    G.write_gguf(p, m)
    r = G.GgufFile(p)
    assert r.metadata["general.architecture"] == "gpt-oss"
    for name, t in m.tensors.items():
        assert r.tensors[name].shape == t.shape
        assert np.array_equal(r.data(name), t.raw())
    e = r.expert_slice("blk.0.ffn_gate_exps.weight", 3)
    per = G.raw_size(G.MXFP4, 256 * 256)
    assert np.array_equal(e, m.tensors["blk.0.ffn_gate_exps.weight"].raw()[3 * per:4 * per])
    r.close()


def _sample_reference_f32(lg, counts, T, top_p, pen, r):
    """SamplingParams::sample (engine.rs:124-208) step by step in f32 with sequential sums"""
    lg = lg.astype(np.float32).copy()
    if pen != 1.0 and counts is not None:
        for v in np.nonzero(counts)[0]:
            for _ in range(int(counts[v])):
                lg[v] = lg[v] / np.float32(pen) if lg[v] > 0 else lg[v] * np.float32(pen)
    if T == 0:
        return int(np.nonzero(lg == lg.max())[0][-1])   # Iterator::max_by: the last maximum
    if T != 1:
        lg = lg * (np.float32(1) / np.float32(T))
    p = np.exp((lg - lg.max()).astype(np.float64)).astype(np.float32)
    s = np.float32(0)
    for v in p:
        s = np.float32(s + v)
    p = (p / s).astype(np.float32)
    if top_p < 1:
        order = np.argsort(-p, kind="stable")
        c, cut = np.float32(0), len(p)
        for i, j in enumerate(order):
            c = np.float32(c + p[j])
            if c > np.float32(top_p):
                cut = i + 1
                break
        keep = np.zeros(len(p), bool)
        keep[order[:cut]] = True
        p = np.where(keep, p, np.float32(0)).astype(np.float32)
        s = np.float32(0)
        for v in p:
            s = np.float32(s + v)
        p = (p / s).astype(np.float32)
    c = np.float32(0)
    for i, v in enumerate(p):
        c = np.float32(c + v)
        if np.float32(r) < c:
            return i
    return len(p) - 1


def test_sampler_follows_reference_algorithm(orc):  # model/engine.rs:124-208
    """the oracle's sampler (sums exact to 2^-109, rounded once) picks the token the reference's
    sequential-f32 algorithm picks: penalties, greedy ties, temperature, top-p, the draw"""
    rng = np.random.default_rng(0)
    for t in range(240):
        V = int(rng.integers(2, 300))
        lg = (rng.standard_normal(V) * 3).astype(np.float32)
        if t % 5 == 0:
            lg[rng.integers(0, V, 4)] = lg.max()   # ties at the maximum
        counts = rng.integers(0, 3, V).astype(np.uint32) if t % 3 == 0 else None
        T = [0.0, 1.0, 0.7, 1.5][t % 4]
        top_p = [1.0, 0.9, 0.5, 0.05][(t // 4) % 4]
        pen = [1.0, 1.3][(t // 16) % 2]
        r = float(rng.random())
        assert orc.sample(lg, counts, T, top_p, pen, r) == _sample_reference_f32(lg, counts, T, top_p, pen, r), t


def test_sampler_edges(orc):
    lg = np.array([1.0, 3.0, 3.0, -2.0], np.float32)
    assert orc.sample(lg, None, 0.0) == 2                     # greedy: the last of equal maxima
    assert orc.sample(lg, np.array([0, 0, 1, 0], np.uint32), 0.0, penalty=2.0) == 1   # 3 / 2 < 3
    assert orc.sample(lg, None, 1.0, top_p=1e-6, r=0.999) == 1  # nucleus of one: the first of the tied maxima
    assert orc.sample(np.zeros(10, np.float32), None, 1.0, top_p=0.35, r=0.99) == 3   # 4 equal tokens kept
    assert orc.sample(lg, None, 1.0, r=0.0) == 0              # the first token with mass
