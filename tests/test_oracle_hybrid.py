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
