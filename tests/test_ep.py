"""Expert parallelism.

CPU (gloo, world size 2): the decomposition the CUDA path uses — each rank combines only its
contiguous expert slice [rank*E/N, (rank+1)*E/N), then a sum all-reduce — reproduces the
single-device MoE layer (oracle, routing over all experts on every rank).

GPU (2 devices): a tiny GPT-OSS-shaped model split over two ranks through the C ABI decodes the
same greedy tokens as one device, with the MoE exchange as an in-graph NCCL all-reduce
(ms_model_init_ep) and as direct stores into the peers' mailboxes over NVLink (ms_model_ep_connect).
"""
import os
import socket
import tempfile

import numpy as np
import pytest

from moe_stream_b200 import synth

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _layer(spec, seed):
    m = synth.build_model(spec, seed)
    t = lambda n: m.tensors["blk.0." + n]
    f = lambda n: t(n).data.astype(np.float32)
    return dict(hidden=spec.hidden, inter=spec.inter, n_experts=spec.experts, top_k=spec.top_k,
                gate_q=spec.expert_gate_q, up_q=spec.expert_gate_q, down_q=spec.expert_down_q,
                gate=t("ffn_gate_exps.weight").raw(), up=t("ffn_up_exps.weight").raw(),
                down=t("ffn_down_exps.weight").raw(), gate_bias=f("ffn_gate_exps.bias"),
                up_bias=f("ffn_up_exps.bias"), down_bias=f("ffn_down_exps.bias"),
                router_w=f("ffn_gate_inp.weight"), router_b=f("ffn_gate_inp.bias"), oai_swiglu=1, norm_topk_prob=1)


def _cpu_rank(rank, world, port, out_path):
    import torch
    import torch.distributed as dist
    from oracle import oracle
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    spec = synth.TINY_GPT_OSS
    L = _layer(spec, 4)
    rng = np.random.default_rng(8)
    x = rng.standard_normal((3, spec.hidden)).astype(np.float32)
    per = spec.experts // world
    local, _, _ = oracle.moe_forward(L, x, expert_range=(rank * per, (rank + 1) * per))
    t = torch.from_numpy(local.copy())
    dist.all_reduce(t)
    if rank == 0:
        np.save(out_path, t.numpy())
    dist.destroy_process_group()


def test_ep_decomposition_gloo(orc, tmp_path):
    import torch.multiprocessing as mp
    out = str(tmp_path / "ep.npy")
    mp.spawn(_cpu_rank, args=(2, _free_port(), out), nprocs=2, join=True)
    spec = synth.TINY_GPT_OSS
    L = _layer(spec, 4)
    x = np.random.default_rng(8).standard_normal((3, spec.hidden)).astype(np.float32)
    full, _, _ = orc.moe_forward(L, x)
    got = np.load(out)
    assert np.abs(got - full).max() / np.abs(full).max() < 1e-5


def _hybrid_layer(seed):
    spec = synth.TINY_QWEN3_NEXT
    m = synth.build_model(spec, seed, only=lambda n: n.startswith("blk.0.ffn"))
    t = lambda n: m.tensors["blk.0." + n]
    L = dict(hidden=spec.hidden, inter=spec.inter, n_experts=spec.experts, top_k=spec.top_k,
             gate_q=spec.expert_gate_q, up_q=spec.expert_gate_q, down_q=spec.expert_down_q,
             gate=t("ffn_gate_exps.weight").raw(), up=t("ffn_up_exps.weight").raw(),
             down=t("ffn_down_exps.weight").raw(), router_w=t("ffn_gate_inp.weight").data.astype(np.float32),
             oai_swiglu=0, norm_topk_prob=1)
    sh = (t("ffn_gate_shexp.weight"), t("ffn_up_shexp.weight"), t("ffn_down_shexp.weight"),
          t("ffn_gate_inp_shexp.weight").data.astype(np.float32))
    return spec, L, sh


def _shared(orc, spec, sh, x, y):
    g, u, d, gi = sh
    return orc.shared_expert(g.qtype, g.raw(), u.raw(), d.qtype, d.raw(), gi, spec.hidden, spec.shared_inter, x, y)


def _cpu_rank_hybrid(rank, world, port, out_path):
    import torch
    import torch.distributed as dist
    from oracle import oracle
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    spec, L, sh = _hybrid_layer(6)
    x = np.random.default_rng(9).standard_normal(spec.hidden).astype(np.float32)
    per = spec.experts // world
    local, _, _ = oracle.moe_forward(L, x, expert_range=(rank * per, (rank + 1) * per))
    t = torch.from_numpy(local.reshape(-1).copy())
    dist.all_reduce(t)                                       # the routed experts' exchange
    out = _shared(oracle, spec, sh, x, t.numpy().copy())     # the replicated shared expert, on every rank
    np.save(out_path.replace(".npy", f"{rank}.npy"), out)
    dist.destroy_process_group()


def test_ep_decomposition_hybrid_gloo(orc, tmp_path):
    """configs[3]'s partition on CPU ranks: 64 experts top-10 split over 2 ranks, shared expert
    replicated and added after the routed exchange; every rank ends with the one-device layer"""
    import torch.multiprocessing as mp
    out = str(tmp_path / "hy.npy")
    mp.spawn(_cpu_rank_hybrid, args=(2, _free_port(), out), nprocs=2, join=True)
    spec, L, sh = _hybrid_layer(6)
    x = np.random.default_rng(9).standard_normal(spec.hidden).astype(np.float32)
    full, idx, _ = orc.moe_forward(L, x)
    assert len(set(idx[0].tolist()) & set(range(spec.experts // 2))) not in (0, spec.top_k)   # both ranks work
    want = _shared(orc, spec, sh, x, full.reshape(-1).copy())
    for r in range(2):
        got = np.load(str(tmp_path / f"hy{r}.npy"))
        assert np.abs(got - want).max() / np.abs(want).max() < 1e-5


def _gpu_rank(rank, world, port, path, prompt, out_dir, exchange, n_new=16):
    import torch
    import torch.distributed as dist
    from moe_stream_b200.engine import Context, Engine
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    ctx = Context(rank)
    eng = Engine.open(path, max_seq_len=256, ep_rank=rank, ep_size=world, ctx=ctx)
    if exchange == "p2p":
        eng.init_ep_p2p()
    else:
        uid = [Engine.nccl_unique_id(ctx) if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        eng.init_ep(uid[0])
    eng.set_prefill(0)   # the prompt through the decode step, as on one device
    toks = eng.generate(prompt, n_new)
    np.save(os.path.join(out_dir, f"tok{rank}.npy"), np.array(toks, np.int32))
    eng.close()
    ctx.close()
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("exchange", ["nccl", "p2p"])
def test_ep_two_gpus_greedy_tokens(tmp_path, exchange):
    import torch
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    f = np.load(os.path.join(GOLD, "tiny_models.npz"))
    path = str(tmp_path / "tiny.gguf")
    synth.write_model(path, synth.TINY_GPT_OSS, seed=7)
    mp.spawn(_gpu_rank, args=(2, _free_port(), path, f["tiny_gpt_oss_prompt"], str(tmp_path), exchange), nprocs=2,
             join=True)
    for r in range(2):
        assert np.load(str(tmp_path / f"tok{r}.npy")).tolist() == f["tiny_gpt_oss_tokens"].tolist()


@pytest.mark.gpu
@pytest.mark.parametrize("exchange", ["p2p", "nccl"])
def test_ep_two_gpus_hybrid_model(tmp_path, exchange):
    """configs[3]'s partition at small scale: the tiny Qwen3-Next hybrid (64 experts top-10, shared
    expert, DeltaNet and gated-attention layers replicated) split 32 + 32 experts over two GPUs
    decodes the one-device oracle's greedy tokens (tests/golden/tiny_qwen3_next.npz)"""
    import torch
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    f = np.load(os.path.join(GOLD, "tiny_qwen3_next.npz"))
    path = str(tmp_path / "hyb.gguf")
    synth.write_model(path, synth.TINY_QWEN3_NEXT, seed=11)
    mp.spawn(_gpu_rank, args=(2, _free_port(), path, f["prompt"], str(tmp_path), exchange, 16), nprocs=2, join=True)
    for r in range(2):
        assert np.load(str(tmp_path / f"tok{r}.npy")).tolist() == f["tokens"][:16].tolist()
