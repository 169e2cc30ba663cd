"""Python host API mirroring moe-stream-core's Engine and its Metal kernel seam.

``Context`` wraps ``ms_ctx`` and exposes the per-dispatch kernels (the functions of
moe-stream-core/src/metal/mod.rs the CUDA backend replaces) on device pointers, so they
can be driven with torch CUDA tensors.  ``Engine`` wraps ``ms_model`` with the reference
Engine's surface (model/engine.rs: ``open_with_device`` 277-598, ``preload_weights`` 1551,
``forward`` 1869-2006, ``generate`` 2011-2118, ``clear_cache`` 2402).  All compute runs in
the CUDA library; nothing here computes on the CPU.
"""
from __future__ import annotations

import ctypes as C
import weakref
from typing import Optional, Sequence

import numpy as np

from . import gguf as G
from ._lib import ARCH_GPT_OSS, ARCH_QWEN_MOE, ModelConfig, check, lib


def _ptr(t) -> int:
    """Device pointer of a torch tensor / raw int / None."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


class Context:
    """One GPU (``Device::new_cuda``); not thread-safe, like the reference Engine."""

    def __init__(self, device: int = 0, stream=None):
        h = C.c_void_p()
        check(lib().ms_ctx_create(device, C.byref(h)))
        self.h = h
        self.device = device
        self._engines = weakref.WeakSet()   # closed before the context (their handles die with it)
        if stream is not None:
            self.set_stream(stream)

    def set_stream(self, stream) -> None:
        """Enqueue on a caller stream (a torch.cuda.Stream or raw cudaStream_t int)."""
        s = getattr(stream, "cuda_stream", stream)
        check(lib().ms_ctx_set_stream(self.h, s), self.h)

    def sync(self) -> None:
        check(lib().ms_sync(self.h), self.h)

    def error_flags(self, clear: bool = True) -> int:
        f = C.c_uint32()
        check(lib().ms_ctx_error_flags(self.h, C.byref(f), int(clear)), self.h)
        return f.value

    @property
    def sm_count(self) -> int:
        return lib().ms_ctx_sm_count(self.h)

    # ---- metal/mod.rs seam ----
    def dequantize(self, qtype: int, blocks, n: int, out) -> None:
        check(lib().ms_dequantize(self.h, qtype, _ptr(blocks), n, _ptr(out)), self.h)

    def rms_norm(self, x, w, y, rows: int, dim: int, eps: float) -> None:
        check(lib().ms_rms_norm(self.h, _ptr(x), _ptr(w), _ptr(y), rows, dim, eps), self.h)

    def gemv(self, qtype: int, w, rows: int, cols: int, x, y, bias=None) -> None:
        check(lib().ms_gemv(self.h, qtype, _ptr(w), rows, cols, _ptr(x), _ptr(bias), _ptr(y)), self.h)

    def router_topk(self, h, norm_w, eps, router_w, router_b, mask, hidden, n_experts, top_k, arch,
                    norm_topk_prob, xn, logits, idx, wts) -> None:
        check(lib().ms_router_topk(self.h, _ptr(h), _ptr(norm_w), eps, _ptr(router_w), _ptr(router_b), _ptr(mask),
                                   hidden, n_experts, top_k, arch, int(norm_topk_prob), _ptr(xn), _ptr(logits),
                                   _ptr(idx), _ptr(wts)), self.h)

    def moe_mxfp4_decode(self, gate, up, down, gate_b, up_b, down_b, hidden, inter, n_experts, top_k, arch,
                         x, idx, wts, h) -> None:
        check(lib().ms_moe_mxfp4_decode(self.h, _ptr(gate), _ptr(up), _ptr(down), _ptr(gate_b), _ptr(up_b),
                                        _ptr(down_b), hidden, inter, n_experts, top_k, arch, _ptr(x), _ptr(idx),
                                        _ptr(wts), _ptr(h)), self.h)

    def moe_mxfp4_decode_noalloc(self, gate, up, down, gate_b, up_b, down_b, hidden, inter, n_experts, top_k,
                                 arch, x, idx, wts, h) -> None:
        """Same as moe_mxfp4_decode, with its scratch in the library's fixed device array."""
        check(lib().ms_moe_mxfp4_decode_noalloc(self.h, _ptr(gate), _ptr(up), _ptr(down), _ptr(gate_b),
                                                _ptr(up_b), _ptr(down_b), hidden, inter, n_experts, top_k, arch,
                                                _ptr(x), _ptr(idx), _ptr(wts), _ptr(h)), self.h)

    @staticmethod
    def mxfp4_packed_bytes(hidden: int, inter: int, n_experts: int):
        """(gate_up_bytes, down_bytes) of the tensor-core expert layout."""
        g, d = C.c_size_t(), C.c_size_t()
        check(lib().ms_mxfp4_packed_bytes(hidden, inter, n_experts, C.byref(g), C.byref(d)))
        return g.value, d.value

    def mxfp4_pack_experts(self, gate, up, down, hidden, inter, n_experts, gu_packed, down_packed) -> None:
        check(lib().ms_mxfp4_pack_experts(self.h, _ptr(gate), _ptr(up), _ptr(down), hidden, inter, n_experts,
                                          _ptr(gu_packed), _ptr(down_packed)), self.h)

    def moe_mxfp4_decode_packed(self, gu_packed, down_packed, gate_b, up_b, down_b, hidden, inter, n_experts, top_k,
                                arch, x, idx, wts, h) -> None:
        """The expert FFN on the tensor cores over packed experts (see mxfp4_pack_experts)."""
        check(lib().ms_moe_mxfp4_decode_packed(self.h, _ptr(gu_packed), _ptr(down_packed), _ptr(gate_b), _ptr(up_b),
                                               _ptr(down_b), hidden, inter, n_experts, top_k, arch, _ptr(x),
                                               _ptr(idx), _ptr(wts), _ptr(h)), self.h)

    def moe_mxfp4_prefill_packed(self, gu_packed, down_packed, gate_b, up_b, down_b, hidden, inter, n_experts,
                                 top_k, arch, x, n_tokens, idx, wts, out, precise: bool = False) -> None:
        """Batched prefill of one MoE layer: grouped bf16 GEMM on the tensor cores (out = MoE(x));
        precise: activations as bf16 hi + lo pairs."""
        check(lib().ms_moe_mxfp4_prefill_packed(self.h, _ptr(gu_packed), _ptr(down_packed), _ptr(gate_b), _ptr(up_b),
                                                _ptr(down_b), hidden, inter, n_experts, top_k, arch, _ptr(x),
                                                n_tokens, _ptr(idx), _ptr(wts), _ptr(out), int(bool(precise))), self.h)

    def rope(self, x, cos, sin, n_tokens: int, heads: int, head_dim: int, rot_dim: int, y) -> None:
        """y = RoPE(x) with per-token cos/sin rows (fused_rope_metal, metal/mod.rs:383-472)."""
        check(lib().ms_rope(self.h, _ptr(x), _ptr(cos), _ptr(sin), n_tokens, heads, head_dim, rot_dim, _ptr(y)),
              self.h)

    def sample(self, logits, counts, temperature: float, top_p: float, repetition_penalty: float, r: float,
               work, token) -> None:
        """token[0] = SamplingParams::sample (engine.rs:124-208) of device logits [V] (f32), with
        counts [V] (uint32, times each token was generated; None = no penalty), draw r in [0, 1)
        and work [V] f32 scratch."""
        check(lib().ms_sample(self.h, _ptr(logits), int(logits.numel()), _ptr(counts) if counts is not None else None,
                              float(temperature), float(top_p), float(repetition_penalty), float(r), _ptr(work),
                              _ptr(token)), self.h)

    def attn_layer_decode(self, layer: dict, pos: int, h) -> None:
        """h += attention(RMSNorm(h)) for one token at `pos` (layer.rs:511-749).  layer: ints hidden,
        heads, kv_heads, head_dim, rot_dim, window, cap, float eps and device tensors attn_norm, wqkv,
        wo, k_cache, v_cache, cos_t, sin_t (bqkv, bo, sinks, q_norm, k_norm, q_gate optional)."""
        from ._lib import AttnLayer
        d = layer
        L = AttnLayer(d["hidden"], d["heads"], d["kv_heads"], d["head_dim"], d["rot_dim"], d["eps"],
                      d.get("window", 0), d["cap"], _ptr(d["attn_norm"]), _ptr(d["wqkv"]), _ptr(d.get("bqkv")),
                      _ptr(d["wo"]), _ptr(d.get("bo")), _ptr(d.get("sinks")), _ptr(d.get("q_norm")),
                      _ptr(d.get("k_norm")), _ptr(d["k_cache"]), _ptr(d["v_cache"]), _ptr(d["cos_t"]),
                      _ptr(d["sin_t"]), int(d.get("q_gate", 0)))
        check(lib().ms_attn_layer_decode(self.h, C.byref(L), pos, _ptr(h)), self.h)

    def deltanet_decode(self, layer: dict, x, conv_state, rec_state, y) -> None:
        """One Gated DeltaNet decode token.  layer: ints hidden, n_k_heads, head_k_dim, n_v_heads,
        head_v_dim, conv_kernel, eps, qkv_q, gate_q, ba_q, out_q and device tensors qkv, gate, ba, out,
        conv1d, ssm_a, dt_bias, norm.  conv_state / rec_state are updated in place; y = layer output."""
        from ._lib import DeltaNetLayer
        d = layer
        L = DeltaNetLayer(d["hidden"], d["n_k_heads"], d["head_k_dim"], d["n_v_heads"], d["head_v_dim"],
                          d["conv_kernel"], d["eps"], d["qkv_q"], _ptr(d["qkv"]), d["gate_q"], _ptr(d["gate"]),
                          d["ba_q"], _ptr(d["ba"]), d["out_q"], _ptr(d["out"]), _ptr(d["conv1d"]),
                          _ptr(d["ssm_a"]), _ptr(d["dt_bias"]), _ptr(d["norm"]))
        check(lib().ms_deltanet_decode(self.h, C.byref(L), _ptr(x), _ptr(conv_state), _ptr(rec_state), _ptr(y)),
              self.h)

    def shared_expert(self, gu_qtype, gate, up, down_qtype, down, gate_inp, hidden, inter, x, y) -> None:
        """y += sigmoid(x . gate_inp) * down(silu(gate x) * up x) for one token (gate_inp may be None)."""
        check(lib().ms_shared_expert(self.h, gu_qtype, _ptr(gate), _ptr(up), down_qtype, _ptr(down), _ptr(gate_inp),
                                     hidden, inter, _ptr(x), _ptr(y)), self.h)

    def close(self) -> None:
        if getattr(self, "h", None):
            for e in list(getattr(self, "_engines", ())):
                e.close()
            lib().ms_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def config_from_model(m: G.Model, max_seq_len: int, ep_rank: int = 0, ep_size: int = 1) -> ModelConfig:
    """config.rs:253-434 for an in-memory GGUF model (same keys and defaults as the file loader)."""
    meta = {k: v for k, (_, v) in m.metadata.items()}
    a = meta.get("general.architecture", "qwen2moe")
    gi = lambda k, d: int(meta.get(f"{a}.{k}", d))
    gf = lambda k, d: float(meta.get(f"{a}.{k}", d))
    c = ModelConfig()
    c.arch = ARCH_GPT_OSS if a == "gpt-oss" else ARCH_QWEN_MOE
    c.hidden = gi("embedding_length", 2048)
    c.layers = gi("block_count", 48)
    c.heads = gi("attention.head_count", 16)
    c.kv_heads = gi("attention.head_count_kv", 2)
    c.head_dim = gi("attention.key_length", c.hidden // c.heads)
    c.experts = gi("expert_count", 128)
    c.top_k = gi("expert_used_count", 8)
    c.inter = gi("expert_feed_forward_length", 768)
    c.vocab = gi("vocab_size", m.tensors["token_embd.weight"].shape[0] if "token_embd.weight" in m.tensors else 151936)
    c.rope_theta = gf("rope.freq_base", 1e6)
    c.eps = gf("attention.layer_norm_rms_epsilon", 1e-6)
    c.sliding_window = gi("attention.sliding_window", 0)
    # partial rotary: rope.partial_rotary_factor, else rope.dimension_count / head_dim (config.rs:328-335)
    prf = meta.get(f"{a}.rope.partial_rotary_factor")
    if prf is None:
        dc = meta.get(f"{a}.rope.dimension_count")
        prf = float(np.float32(dc) / np.float32(c.head_dim)) if dc is not None else 1.0
    c.rot_dim = int(np.float32(c.head_dim) * np.float32(prf))
    # DeltaNet hybrids (config.rs:318-352): SSM tensors imply an attention interval of 4
    has_ssm = "blk.0.ssm_a" in m.tensors or "blk.0.ssm_conv1d.weight" in m.tensors
    c.attn_interval = gi("attention.full_attention_interval", 4 if has_ssm else 0)
    c.ssm_groups = gi("ssm.group_count", 16)
    c.ssm_state = gi("ssm.state_size", 128)
    c.ssm_dt_rank = int(meta.get(f"{a}.ssm.time_step_rank", meta.get(f"{a}.ssm.dt_rank", 32)))
    c.ssm_inner = gi("ssm.inner_size", 4096)
    c.ssm_conv = gi("ssm.conv_kernel", 4)
    name = meta.get("general.name", "")
    c.norm_topk_prob = int(not ("Qwen1.5" in name or "Qwen2" in name))
    c.max_seq_len = max_seq_len
    c.ep_rank, c.ep_size = ep_rank, ep_size
    c.attn_splits = 0
    return c


class Engine:
    """GPU-resident engine over one GGUF model (the reference's GpuResident mode)."""

    def __init__(self, handle: C.c_void_p, ctx: Context):
        self.h = handle
        self.ctx = ctx
        ctx._engines.add(self)
        cfg = ModelConfig()
        check(lib().ms_model_get_config(self.h, C.byref(cfg)), ctx.h)
        self.config = cfg

    # engine.rs:277 open_with_device
    @classmethod
    def open(cls, path: str, max_seq_len: int = 4096, device: int = 0, ep_rank: int = 0, ep_size: int = 1,
             ctx: Optional[Context] = None, expert_slots: int = 0) -> "Engine":
        """expert_slots > 0: host-tier experts (pinned host memory, an HBM LRU of that many experts per
        layer; the reference's SSD-streaming mode)."""
        ctx = ctx or Context(device)
        h = C.c_void_p()
        if expert_slots > 0:
            if ep_size != 1:
                raise ValueError("host-tier experts run on one GPU")
            check(lib().ms_model_open_gguf_tiered(ctx.h, path.encode(), max_seq_len, expert_slots, C.byref(h)), ctx.h)
        else:
            check(lib().ms_model_open_gguf(ctx.h, path.encode(), max_seq_len, ep_rank, ep_size, C.byref(h)), ctx.h)
        return cls(h, ctx)

    def set_dynamic_k(self, enable: bool, k_min: int = 2, k_max: int = 0, layer_adaptive: bool = False) -> None:
        """per-step K from router entropy (layer.rs:947-1011); k_max 0 = the model's top_k"""
        check(lib().ms_model_set_dynamic_k(self.h, int(enable), k_min, k_max or self.config.top_k,
                                           int(layer_adaptive)), self.ctx.h)

    def set_router_stats(self, enable: bool) -> None:
        check(lib().ms_model_set_router_stats(self.h, int(enable)), self.ctx.h)

    def router_stats(self):
        """(router entropy [layers], K routed [layers]) of the last step"""
        n = self.config.layers
        ent = np.empty(n, np.float32)
        k = np.empty(n, np.int32)
        check(lib().ms_model_router_stats(self.h, ent.ctypes.data_as(C.POINTER(C.c_float)),
                                          k.ctypes.data_as(C.POINTER(C.c_int32))), self.ctx.h)
        return ent, k

    def router_totals(self, max_steps: int = 4096) -> dict:
        """Running routing statistics since set_router_stats(True), with the reference's summaries
        (RoutingStatsCollector::summary and EntropyProfiler::summary, model/cache.rs:404-580):
        counts / weight_sums [layers, experts], tokens [layers], entropy_log [steps, layers],
        frequency, mean_gate_weight, importance [layers, experts] (f64) and per-layer entropy
        mean / std / min / max (f32, as the reference accumulates them)."""
        c = self.config
        counts = np.zeros((c.layers, c.experts), np.uint64)
        wsum = np.zeros((c.layers, c.experts), np.float64)
        tokens = np.zeros(c.layers, np.uint64)
        log = np.zeros((max_steps, c.layers), np.float32)
        n = C.c_int()
        check(lib().ms_model_router_totals(self.h, counts.ctypes.data, wsum.ctypes.data, tokens.ctypes.data,
                                           log.ctypes.data, max_steps, C.byref(n)), self.ctx.h)
        log = log[:min(n.value, max_steps)]
        freq = np.where(tokens[:, None] > 0, counts / np.maximum(tokens[:, None], 1).astype(np.float64), 0.0)
        mean_w = np.where(counts > 0, wsum / np.maximum(counts, 1).astype(np.float64), 0.0)
        ent = {"mean": [], "std": [], "min": [], "max": []}
        for li in range(c.layers):
            v = log[:, li]
            if v.size == 0:
                for key in ent:
                    ent[key].append(0.0)
                continue
            nf = np.float32(v.size)
            mean = np.float32(0.0)
            for x in v:   # f32 running sums, as the reference's iterator sums
                mean = np.float32(mean + x)
            mean = np.float32(mean / nf)
            var = np.float32(0.0)
            for x in v:
                var = np.float32(var + np.float32(np.float32(x - mean) ** 2))
            ent["mean"].append(float(mean))
            ent["std"].append(float(np.sqrt(np.float32(var / nf))))
            ent["min"].append(float(v.min()))
            ent["max"].append(float(v.max()))
        return dict(counts=counts, weight_sums=wsum, tokens=tokens, entropy_log=log, frequency=freq,
                    mean_gate_weight=mean_w, importance=freq * mean_w, entropy=ent, steps=n.value)

    def expert_tier_stats(self):
        """(hits, misses) of the host-tier expert slots"""
        hits, misses = C.c_uint64(), C.c_uint64()
        check(lib().ms_model_expert_tier_stats(self.h, C.byref(hits), C.byref(misses)), self.ctx.h)
        return hits.value, misses.value

    @classmethod
    def from_model(cls, m: G.Model, max_seq_len: int = 4096, device: int = 0, ep_rank: int = 0, ep_size: int = 1,
                   ctx: Optional[Context] = None, attn_splits: int = 0, expert_slots: int = 0) -> "Engine":
        """Upload an in-memory GGUF model (native block layouts) without writing a file."""
        ctx = ctx or Context(device)
        cfg = config_from_model(m, max_seq_len, ep_rank, ep_size)
        cfg.attn_splits = attn_splits
        h = C.c_void_p()
        check(lib().ms_model_create(ctx.h, C.byref(cfg), C.byref(h)), ctx.h)
        try:
            if expert_slots:
                check(lib().ms_model_set_expert_tier(h, expert_slots), ctx.h)
            for name, t in m.tensors.items():
                raw = t.raw()
                dims = (C.c_int64 * len(t.shape))(*t.shape)
                check(lib().ms_model_set_tensor(h, name.encode(), t.qtype, len(t.shape), dims, raw.ctypes.data,
                                                raw.size), ctx.h)
            check(lib().ms_model_finalize(h), ctx.h)
        except Exception:
            lib().ms_model_destroy(h)
            raise
        return cls(h, ctx)

    @classmethod
    def from_spec(cls, spec, seed: int = 0, max_seq_len: int = 4096, device: int = 0, ep_rank: int = 0,
                  ep_size: int = 1, ctx: Optional[Context] = None, attn_splits: int = 0,
                  progress=None, share=None) -> "Engine":
        """Generate a seeded synthetic model tensor by tensor and upload each as it is made,
        so host memory holds one tensor at a time (the benchmark's 13 GB GPT-OSS shape).
        share(name) -> name or None: tensors mapped to the same name get the bytes generated once for
        that name (each is still uploaded to its own device buffer), e.g. one set of expert stacks for
        every layer of a 43 GB model whose generation would otherwise dominate the run."""
        from . import synth
        ctx = ctx or Context(device)
        meta = G.Model()
        for k, (vt, v) in synth.metadata(spec).items():
            meta.add_meta(k, vt, v)
        cfg = config_from_model(meta, max_seq_len, ep_rank, ep_size)
        cfg.attn_splits = attn_splits
        h = C.c_void_p()
        check(lib().ms_model_create(ctx.h, C.byref(cfg), C.byref(h)), ctx.h)
        try:
            shared = {}
            for name, q, shape, gen in synth.tensor_defs(spec):
                key = share(name) if share else None
                if key is not None and key in shared:
                    raw = shared[key]
                else:
                    raw = np.ascontiguousarray(gen(synth.tensor_rng(seed, key or name))).view(np.uint8).reshape(-1)
                    if key is not None:
                        shared[key] = raw
                dims = (C.c_int64 * len(shape))(*shape)
                check(lib().ms_model_set_tensor(h, name.encode(), q, len(shape), dims, raw.ctypes.data, raw.size),
                      ctx.h)
                if progress:
                    progress(name)
                del raw
            check(lib().ms_model_finalize(h), ctx.h)
        except Exception:
            lib().ms_model_destroy(h)
            raise
        return cls(h, ctx)

    @staticmethod
    def nccl_unique_id(ctx: Context) -> bytes:
        """128-byte NCCL id for an expert-parallel group (rank 0 makes it, every rank receives it)."""
        buf = (C.c_uint8 * 128)()
        check(lib().ms_nccl_unique_id(ctx.h, buf, 128), ctx.h)
        return bytes(buf)

    def init_ep(self, unique_id: bytes) -> None:
        """Join the expert-parallel group (all-reduce of each layer's MoE output)."""
        buf = (C.c_uint8 * 128).from_buffer_copy(unique_id[:128])
        check(lib().ms_model_init_ep(self.h, buf, 128), self.ctx.h)

    def ep_handle(self) -> bytes:
        """This rank's peer-memory mailbox handle (CUDA IPC, 64 bytes)."""
        buf = (C.c_uint8 * 64)()
        check(lib().ms_model_ep_handle(self.h, buf, 64), self.ctx.h)
        return bytes(buf)

    def ep_connect(self, handles: Sequence[bytes]) -> None:
        """Open every rank's mailbox (handles in rank order): the MoE exchange then runs over
        NVLink peer memory instead of NCCL."""
        b = b"".join(handles)
        buf = (C.c_uint8 * len(b)).from_buffer_copy(b)
        check(lib().ms_model_ep_connect(self.h, buf, len(b)), self.ctx.h)

    def init_ep_p2p(self) -> None:
        """ep_handle + all-gather over torch.distributed + ep_connect."""
        import torch.distributed as dist
        hs = [None] * dist.get_world_size()
        dist.all_gather_object(hs, self.ep_handle())
        self.ep_connect(hs)

    def preload_weights(self) -> None:
        """Weights are uploaded to HBM at open; nothing to preload (engine.rs:1551)."""

    def warmup_gpu(self) -> None:
        """The decode step is captured as a CUDA graph on its first run (engine.rs:1683)."""

    def forward(self, tokens: Sequence[int]) -> np.ndarray:
        """Tokens at the current position; returns the last position's logits (engine.rs:1869)."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty(self.config.vocab, dtype=np.float32)
        check(lib().ms_model_forward(self.h, t.ctypes.data_as(C.POINTER(C.c_int32)), t.size,
                                     out.ctypes.data_as(C.POINTER(C.c_float))), self.ctx.h)
        return out

    def decode_step(self, token: int) -> int:
        nxt = C.c_int32()
        check(lib().ms_model_decode_step(self.h, int(token), C.byref(nxt)), self.ctx.h)
        return nxt.value

    def generate(self, prompt: Sequence[int], max_new_tokens: int) -> list:
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(max_new_tokens, dtype=np.int32)
        n = C.c_int()
        check(lib().ms_model_generate(self.h, p.ctypes.data_as(C.POINTER(C.c_int32)), p.size, max_new_tokens,
                                      out.ctypes.data_as(C.POINTER(C.c_int32)), C.byref(n)), self.ctx.h)
        return out[:n.value].tolist()

    def decode_steps_device(self, n: int) -> None:
        check(lib().ms_model_decode_steps_device(self.h, n), self.ctx.h)

    def token_log(self) -> list:
        cap = self.config.max_seq_len
        out = np.empty(cap, dtype=np.int32)
        n = C.c_int()
        check(lib().ms_model_token_log(self.h, out.ctypes.data_as(C.POINTER(C.c_int32)), cap, C.byref(n)),
              self.ctx.h)
        return out[:n.value].tolist()

    def clear_cache(self) -> None:
        check(lib().ms_model_clear_cache(self.h), self.ctx.h)

    @property
    def seq_len(self) -> int:
        n = C.c_int()
        check(lib().ms_model_seq_len(self.h, C.byref(n)), self.ctx.h)
        return n.value

    def last_hidden(self) -> np.ndarray:
        o = np.empty(self.config.hidden, dtype=np.float32)
        check(lib().ms_model_last_hidden(self.h, o.ctypes.data_as(C.POINTER(C.c_float))), self.ctx.h)
        return o

    def last_routing(self, layer: int):
        k = self.config.top_k
        idx = np.empty(k, dtype=np.int32)
        w = np.empty(k, dtype=np.float32)
        check(lib().ms_model_last_routing(self.h, layer, idx.ctypes.data_as(C.POINTER(C.c_int32)),
                                          w.ctypes.data_as(C.POINTER(C.c_float))), self.ctx.h)
        return idx, w

    def last_logits(self) -> np.ndarray:
        o = np.empty(self.config.vocab, dtype=np.float32)
        check(lib().ms_model_last_logits(self.h, o.ctypes.data_as(C.POINTER(C.c_float))), self.ctx.h)
        return o

    def set_exact(self, enable: bool) -> None:
        """Order-independent decode numerics (f64 reductions rounded once; default) or the
        pipelined f32 kernels."""
        check(lib().ms_model_set_exact(self.h, int(enable)), self.ctx.h)

    def set_sampling(self, enable: bool, temperature: float = 1.0, top_p: float = 1.0,
                     repetition_penalty: float = 1.0, seed: int = 0) -> None:
        """Draw each step's token on the device (SamplingParams::sample, engine.rs:124-208) instead
        of the greedy argmax; the n-th draw comes from SplitMix64(seed, n)."""
        check(lib().ms_model_set_sampling(self.h, int(enable), float(temperature), float(top_p),
                                          float(repetition_penalty), int(seed) & ((1 << 64) - 1)), self.ctx.h)

    def generate_sampled(self, prompt: Sequence[int], max_new_tokens: int, temperature: float = 1.0,
                         top_p: float = 1.0, repetition_penalty: float = 1.0, seed: int = 0) -> list:
        """Engine::generate_sampled (engine.rs:2222-2300) with a seeded draw; leaves sampling off."""
        self.set_sampling(True, temperature, top_p, repetition_penalty, seed)
        try:
            return self.generate(prompt, max_new_tokens)
        finally:
            self.set_sampling(False)

    def set_prefill(self, mode: int) -> None:
        """Prompt handling of forward(): 1 batched (bf16 hi/lo expert GEMM, default), 2 batched
        (plain bf16), 0 one decode step per token."""
        check(lib().ms_model_set_prefill(self.h, int(mode)), self.ctx.h)

    def set_trace(self, enable: bool) -> None:
        """Copy each layer's output and router logits during later steps (parity diagnostics)."""
        check(lib().ms_model_set_trace(self.h, int(enable)), self.ctx.h)

    def layer_trace(self):
        """(hidden after each layer [layers, H], router logits [layers, E]) of the last step."""
        c = self.config
        hid = np.empty(c.layers * c.hidden, dtype=np.float32)
        lg = np.empty(c.layers * c.experts, dtype=np.float32)
        fp = C.POINTER(C.c_float)
        check(lib().ms_model_layer_trace(self.h, hid.ctypes.data_as(fp), lg.ctypes.data_as(fp)), self.ctx.h)
        return hid.reshape(c.layers, c.hidden), lg.reshape(c.layers, c.experts)

    def set_graph(self, enable: bool) -> None:
        check(lib().ms_model_set_graph(self.h, int(enable)), self.ctx.h)

    def profile_step(self) -> list:
        """Device microseconds of each kernel of one greedy decode step, in launch order."""
        buf = np.empty(4096, dtype=np.float32)
        n = C.c_int()
        check(lib().ms_model_profile_step(self.h, buf.ctypes.data_as(C.POINTER(C.c_float)), buf.size, C.byref(n)),
              self.ctx.h)
        return buf[:n.value].tolist()

    @property
    def kernels_per_step(self) -> int:
        return lib().ms_model_kernels_per_step(self.h)

    # ---- lockstep batch: B sequences at one shared position (forward over input_ids [B, T]) ----
    def batch_open(self, batch: int) -> None:
        check(lib().ms_model_batch_open(self.h, batch), self.ctx.h)
        self.batch = batch

    def batch_close(self) -> None:
        check(lib().ms_model_batch_close(self.h), self.ctx.h)

    def batch_clear(self) -> None:
        check(lib().ms_model_batch_clear(self.h), self.ctx.h)

    def batch_forward(self, tokens) -> list:
        """tokens [B, T]; returns each sequence's greedy next token after the last position"""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        if t.ndim != 2 or t.shape[0] != self.batch:
            raise ValueError(f"tokens must be [{self.batch}, T]")
        nxt = np.empty(self.batch, dtype=np.int32)
        check(lib().ms_model_batch_forward(self.h, t.ctypes.data_as(C.POINTER(C.c_int32)), t.shape[1],
                                           nxt.ctypes.data_as(C.POINTER(C.c_int32))), self.ctx.h)
        return nxt.tolist()

    def batch_decode_steps_device(self, n: int) -> None:
        check(lib().ms_model_batch_decode_steps_device(self.h, n), self.ctx.h)

    def batch_next_tokens(self) -> list:
        nxt = np.empty(self.batch, dtype=np.int32)
        check(lib().ms_model_batch_next_tokens(self.h, nxt.ctypes.data_as(C.POINTER(C.c_int32))), self.ctx.h)
        return nxt.tolist()

    def batch_token_log(self) -> np.ndarray:
        """tokens fed per step, [steps, B]"""
        cap = self.config.max_seq_len
        out = np.empty((cap, self.batch), dtype=np.int32)
        n = C.c_int()
        check(lib().ms_model_batch_token_log(self.h, out.ctypes.data_as(C.POINTER(C.c_int32)), cap, C.byref(n)),
              self.ctx.h)
        return out[:n.value]

    def batch_generate(self, prompts, max_new_tokens: int) -> np.ndarray:
        """Greedy decode of B equal-length prompts in lockstep; returns [B, max_new_tokens]."""
        self.batch_clear()
        p = np.ascontiguousarray(prompts, dtype=np.int32)
        self.batch_forward(p)
        self.batch_decode_steps_device(max_new_tokens - 1)
        last = self.batch_next_tokens()
        log = self.batch_token_log()
        gen = log[p.shape[1]:].T if max_new_tokens > 1 else np.empty((self.batch, 0), np.int32)
        return np.concatenate([gen, np.asarray(last, np.int32)[:, None]], axis=1)

    def batch_last_logits(self) -> np.ndarray:
        o = np.empty((self.batch, self.config.vocab), dtype=np.float32)
        check(lib().ms_model_batch_last_logits(self.h, o.ctypes.data_as(C.POINTER(C.c_float))), self.ctx.h)
        return o

    BATCH_CLASSES = ["step_start", "qkv_q8", "attention", "o_q8", "router", "expert_grouping", "gate_up", "down",
                     "residual", "lm_head"]

    def batch_profile_step(self) -> dict:
        """Device microseconds of each launch class of one batch step, measured alone."""
        buf = np.empty(64, dtype=np.float32)
        n = C.c_int()
        check(lib().ms_model_batch_profile_step(self.h, buf.ctypes.data_as(C.POINTER(C.c_float)), buf.size,
                                                C.byref(n)), self.ctx.h)
        return {k: round(float(v), 1) for k, v in zip(self.BATCH_CLASSES, buf[:n.value])}

    @property
    def batch_kernels_per_step(self) -> int:
        return lib().ms_model_batch_kernels_per_step(self.h)

    def close(self) -> None:
        if getattr(self, "h", None):
            if getattr(self.ctx, "h", None):   # a closed context already freed its models
                lib().ms_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


__all__ = ["Context", "Engine", "config_from_model", "ARCH_GPT_OSS", "ARCH_QWEN_MOE"]
