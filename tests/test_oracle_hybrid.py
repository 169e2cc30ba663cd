"""The C oracle's Gated DeltaNet decode step and shared expert against an independent float64
numpy restatement (model/deltanet.rs:204-543, model/layer.rs:2250-2293).

The reference holds no golden vectors or tests for these blocks, so this cross-check of two
restatements is what pins them: parity for DeltaNet and the shared expert is "unpinned" against
the reference's own outputs."""
import numpy as np
import pytest

from moe_stream_b200 import gguf as G

from . import hybrid_synth as hs


def rel_err(got, want):
    return float(np.abs(np.asarray(got, np.float64) - want).max() / max(np.abs(want).max(), 1e-30))


@pytest.mark.parametrize("shape", [dict(), dict(nk=1, hkd=32, nv=2, ks=3), dict(nk=2, hkd=128, nv=2, ks=1)])
def test_deltanet_oracle_multi_step(orc, shape):
    d = hs.deltanet_layer(7, **shape)
    conv_dim = 2 * d["n_k_heads"] * d["head_k_dim"] + d["n_v_heads"] * d["head_v_dim"]
    cs = np.zeros((conv_dim, d["conv_kernel"] - 1), np.float32)
    rs = np.zeros((d["n_v_heads"], d["head_k_dim"], d["head_v_dim"]), np.float32)
    cs_np, rs_np = cs.copy(), rs.copy()
    rng = np.random.default_rng(1)
    for _ in range(5):
        x = rng.standard_normal(d["hidden"]).astype(np.float32)
        y = orc.deltanet_step(d, x, cs, rs)
        y_np, cs_np, rs_np = hs.deltanet_step_np(orc, d, x, cs_np, rs_np)
        assert rel_err(y, y_np) < 1e-4
        if cs.size:
            assert rel_err(cs, cs_np) < 1e-6
        assert rel_err(rs, rs_np) < 1e-4


def test_deltanet_oracle_kquant(orc):
    d = hs.deltanet_layer(3, qtype=G.Q4_K)
    conv_dim = 2 * d["n_k_heads"] * d["head_k_dim"] + d["n_v_heads"] * d["head_v_dim"]
    cs = np.zeros((conv_dim, 3), np.float32)
    rs = np.zeros((d["n_v_heads"], d["head_k_dim"], d["head_v_dim"]), np.float32)
    x = np.random.default_rng(2).standard_normal(d["hidden"]).astype(np.float32)
    y = orc.deltanet_step(d, x, cs, rs)
    y_np, _, _ = hs.deltanet_step_np(orc, d, x, np.zeros_like(cs), np.zeros_like(rs))
    assert rel_err(y, y_np) < 1e-4


@pytest.mark.parametrize("gated", [True, False])
def test_shared_expert_oracle(orc, gated):
    e = hs.shared_expert(5, gated=gated)
    x = np.random.default_rng(4).standard_normal(e["hidden"]).astype(np.float32)
    y0 = np.random.default_rng(6).standard_normal(e["hidden"]).astype(np.float32)
    y = orc.shared_expert(e["gu_q"], e["gate"], e["up"], e["down_q"], e["down"], e["gate_inp"], e["hidden"],
                          e["inter"], x, y0.copy())
    want = y0.astype(np.float64) + hs.shared_expert_np(orc, e, x)
    assert rel_err(y, want) < 1e-5


# ---- whole hybrid model (config.rs:446-458 layer dispatch, layer.rs:393-503) ----
import os  # noqa: E402

from moe_stream_b200 import synth  # noqa: E402

GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def hybrid(tmp_path_factory):
    spec = synth.TINY_QWEN3_NEXT
    path = str(tmp_path_factory.mktemp("hybrid") / "tiny_qwen3_next.gguf")
    model = synth.build_model(spec, seed=11)
    G.write_gguf(path, model)
    return spec, model, path


def test_hybrid_oracle_matches_its_golden(orc, hybrid):
    """the oracle's hybrid forward is reproducible across machines (fixture made by
    tests/golden/make_hybrid_golden.py)"""
    spec, _, path = hybrid
    f = np.load(os.path.join(GOLD, "tiny_qwen3_next.npz"))
    om = orc.Model(path, max_seq_len=64)
    assert om.generate(f["prompt"], len(f["tokens"])).tolist() == f["tokens"].tolist()
    om.clear_cache()
    assert rel_err(om.forward(f["prompt"]), f["logits"].astype(np.float64)) < 1e-6
    hid, lg = om.layer_trace(spec.layers, spec.experts)
    assert rel_err(hid, f["layer_hidden"].astype(np.float64)) < 1e-6
    om.close()


def _deq(orc, t):
    n = int(np.prod(t.shape))
    return orc.dequantize(t.qtype, t.raw(), n).reshape(t.shape).astype(np.float64)


def _rms(x, w, eps):
    return x / np.sqrt((x * x).mean() + eps) * w


def test_hybrid_layer_dispatch_matches_numpy(orc, hybrid):
    """One token at position 0 through the oracle's hybrid model against a float64 numpy composition
    of the reference's layer: attention every 4th layer (gated Q, output x sigmoid(gate); at one
    position the softmax is 1, so the attention output is V), Gated DeltaNet otherwise (the numpy
    DeltaNet restatement above), then router softmax / top-10 / renormalise, the routed experts in
    ascending order plus the shared expert.  The oracle's Q8_0 projections run in exact-f32 mode here
    so the comparison measures the wiring, not Q8_0 activation rounding."""
    spec, model, path = hybrid
    T = model.tensors
    H, E, K, I, hd = spec.hidden, spec.experts, spec.top_k, spec.inter, spec.head_dim
    nh, nkv = spec.heads, spec.kv_heads
    token = 17
    om = orc.Model(path, max_seq_len=8, attn_mode=0)
    om.forward(np.array([token], np.int32))
    o_hid, o_lg = om.layer_trace(spec.layers, E)
    o_idx, _ = om.last_routing(spec.layers, K)
    om.close()
    emb = T["token_embd.weight"].data.reshape(spec.vocab, H)
    h = emb[token].astype(np.float64)
    for li in range(spec.layers):
        p = f"blk.{li}."
        x = _rms(h, T[p + "attn_norm.weight"].data.astype(np.float64), spec.eps)
        if spec.is_attention_layer(li):
            qg = _deq(orc, T[p + "attn_q.weight"]) @ x
            v = _deq(orc, T[p + "attn_v.weight"]) @ x
            gate = qg.reshape(nh, 2, hd)[:, 1, :]
            att = np.repeat(v.reshape(nkv, hd), nh // nkv, axis=0) / (1.0 + np.exp(-gate))
            y = _deq(orc, T[p + "attn_output.weight"]) @ att.reshape(-1)
        else:
            assert p + "attn_q.weight" not in T
            d = dict(hidden=H, n_k_heads=spec.ssm_groups, head_k_dim=spec.ssm_state, n_v_heads=spec.ssm_dt_rank,
                     head_v_dim=spec.ssm_inner // spec.ssm_dt_rank, conv_kernel=spec.ssm_conv, eps=spec.eps,
                     qkv_q=T[p + "attn_qkv.weight"].qtype, qkv=T[p + "attn_qkv.weight"].raw(),
                     gate_q=T[p + "attn_gate.weight"].qtype, gate=T[p + "attn_gate.weight"].raw(),
                     ba_q=T[p + "ssm_ba.weight"].qtype, ba=T[p + "ssm_ba.weight"].raw(),
                     out_q=T[p + "ssm_out.weight"].qtype, out=T[p + "ssm_out.weight"].raw(),
                     conv1d=T[p + "ssm_conv1d.weight"].data.reshape(-1, spec.ssm_conv),
                     ssm_a=T[p + "ssm_a"].data, dt_bias=T[p + "ssm_dt.bias"].data,
                     norm=T[p + "ssm_norm.weight"].data)
            conv = np.zeros((spec.ssm_conv_dim, spec.ssm_conv - 1), np.float32)
            rec = np.zeros((spec.ssm_dt_rank, spec.ssm_state, spec.ssm_inner // spec.ssm_dt_rank), np.float32)
            y, _, _ = hs.deltanet_step_np(orc, d, x.astype(np.float32), conv, rec)
        h = h + y
        x = _rms(h, T[p + "ffn_norm.weight"].data.astype(np.float64), spec.eps)
        logits = T[p + "ffn_gate_inp.weight"].data.reshape(E, H).astype(np.float64) @ x
        assert rel_err(o_lg[li], logits) < 1e-4
        prob = np.exp(logits - logits.max())
        prob /= prob.sum()
        order = np.argsort(-prob, kind="stable")[:K]
        srt = np.sort(prob)[::-1]
        assert srt[K - 1] - srt[K] > 1e-5, "seed has a near-tie at the top-k boundary"
        assert sorted(order.tolist()) == sorted(o_idx[li].tolist())
        w = prob[order] / prob[order].sum()
        gate = _deq(orc, T[p + "ffn_gate_exps.weight"])
        up = _deq(orc, T[p + "ffn_up_exps.weight"])
        down = _deq(orc, T[p + "ffn_down_exps.weight"])
        moe = np.zeros(H)
        for e, wk in sorted(zip(order.tolist(), w.tolist())):
            g, u = gate[e] @ x, up[e] @ x
            moe += wk * (down[e] @ (g / (1.0 + np.exp(-g)) * u))
        sh = dict(hidden=H, inter=spec.shared_inter, gu_q=T[p + "ffn_gate_shexp.weight"].qtype,
                  gate=T[p + "ffn_gate_shexp.weight"].raw(), up=T[p + "ffn_up_shexp.weight"].raw(),
                  down_q=T[p + "ffn_down_shexp.weight"].qtype, down=T[p + "ffn_down_shexp.weight"].raw(),
                  gate_inp=T[p + "ffn_gate_inp_shexp.weight"].data)
        h = h + moe + hs.shared_expert_np(orc, sh, x.astype(np.float32))
        assert rel_err(o_hid[li], h) < 1e-4, f"layer {li}"
    assert [spec.is_attention_layer(li) for li in range(spec.layers)] == [False, False, False, True] * 2


def test_engine_config_reads_hybrid_keys():
    """host-side GGUF config of the Python binding (config.rs:318-352): interval, ssm shape, partial
    rotary; and the defaults a file without the interval key but with SSM tensors gets"""
    from moe_stream_b200.engine import config_from_model
    spec = synth.TINY_QWEN3_NEXT
    m = synth.build_model(spec, seed=1, only=lambda n: n.startswith("blk.0.") or n == "token_embd.weight")
    c = config_from_model(m, max_seq_len=32)
    assert (c.attn_interval, c.ssm_groups, c.ssm_state, c.ssm_dt_rank, c.ssm_inner, c.ssm_conv) == \
        (4, spec.ssm_groups, spec.ssm_state, spec.ssm_dt_rank, spec.ssm_inner, spec.ssm_conv)
    assert c.rot_dim == int(spec.head_dim * spec.rot_factor) == 64
    del m.metadata[f"{spec.arch}.attention.full_attention_interval"]
    del m.metadata[f"{spec.arch}.rope.partial_rotary_factor"]
    m.add_meta(f"{spec.arch}.rope.dimension_count", G.T_U32, 128)
    c = config_from_model(m, max_seq_len=32)
    assert c.attn_interval == 4 and c.rot_dim == 128   # SSM tensors present: every 4th layer attention
    plain = synth.build_model(synth.TINY_QWEN3, seed=1, only=lambda n: n == "token_embd.weight")
    c = config_from_model(plain, max_seq_len=32)
    assert c.attn_interval == 0 and c.rot_dim == synth.TINY_QWEN3.head_dim
