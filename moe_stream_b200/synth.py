"""Seeded synthetic MoE models in native GGUF block layouts.

Shapes and value distributions are the ones the benchmark configurations name:
GPT-OSS-20B-shaped MXFP4 experts (e2m1 codes uniform over the 16 values, e8m0
scale byte uniform in 119..123, i.e. 2^-8..2^-4), f32 router ~N(0,0.02) with bias
~N(0,0.01), Q8_0 attention projections quantized from ~N(0,0.02), f16 embedding
and LM head ~N(0,0.02); Qwen3-30B-A3B-shaped models with Q4_K gate/up and Q6_K
down experts whose sub-block scales/mins are uniform over their valid ranges.

Every tensor is generated from its own generator seeded by (model seed, tensor
name), so any subset of a model can be regenerated independently and the same
bytes come out on every machine.  Tensor names and metadata keys follow the GGUF
conventions that moe-stream-core reads (config.rs:253-434, layer.rs:393-744,
engine.rs:354-361, engine.rs:606-921).
"""
from __future__ import annotations

import hashlib
from dataclasses import dataclass, replace
from typing import Callable, Dict, Iterator, Optional, Tuple

import numpy as np

from . import gguf as G


@dataclass(frozen=True)
class ModelSpec:
    arch: str = "gpt-oss"           # "gpt-oss" (OAI SwiGLU, softmax over top-k) or "qwen3moe"
    name: str = "synthetic"
    hidden: int = 2880
    layers: int = 24
    heads: int = 64
    kv_heads: int = 8
    head_dim: int = 64
    experts: int = 32
    top_k: int = 4
    inter: int = 2880
    vocab: int = 201088
    rope_theta: float = 150000.0
    eps: float = 1e-5
    sliding_window: int = 128       # 0 = none; even layers are SWA when > 0
    expert_gate_q: int = G.MXFP4
    expert_down_q: int = G.MXFP4
    attn_q: int = G.Q8_0
    embed_q: int = G.F16
    expert_bias: bool = True
    attn_bias: bool = True
    sinks: bool = True
    qk_norm: bool = False
    router_bias: bool = True
    with_attention: bool = True     # False: MoE-only layer stack (config 0)
    with_lm: bool = True            # embedding / final norm / LM head present
    # DeltaNet hybrids (Qwen3-Next): layer l is gated attention when (l + 1) % attn_interval == 0,
    # else Gated DeltaNet with ssm_groups k heads of ssm_state dims, ssm_dt_rank v heads of
    # ssm_inner / ssm_dt_rank dims and a causal conv of ssm_conv taps (config.rs:318-352, 446-494)
    attn_interval: int = 0
    ssm_groups: int = 16
    ssm_state: int = 128
    ssm_dt_rank: int = 32
    ssm_inner: int = 4096
    ssm_conv: int = 4
    ssm_q: int = G.Q4_K             # DeltaNet projections (attn_qkv, attn_gate, ssm_ba, ssm_out)
    shared_inter: int = 0           # > 0: one always-on shared expert of this width per layer
    shared_q: int = G.Q4_K
    rot_factor: float = 1.0         # rope.partial_rotary_factor (rotary dims = head_dim * factor)

    @property
    def q_dim(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim

    def is_attention_layer(self, layer: int) -> bool:
        return self.attn_interval == 0 or (layer + 1) % self.attn_interval == 0

    @property
    def ssm_conv_dim(self) -> int:
        return 2 * self.ssm_groups * self.ssm_state + self.ssm_inner


# ---- named configurations -------------------------------------------------
GPT_OSS_20B = ModelSpec()
# one GPT-OSS MoE FFN layer, no attention, no embedding
GPT_OSS_MOE_LAYER = replace(GPT_OSS_20B, layers=1, with_attention=False, with_lm=False)
QWEN3_30B_A3B = ModelSpec(arch="qwen3moe", name="Qwen3-30B-A3B-synthetic", hidden=2048, layers=48,
                          heads=32, kv_heads=4, head_dim=128, experts=128, top_k=8, inter=768,
                          vocab=151936, rope_theta=1e6, eps=1e-6, sliding_window=0,
                          expert_gate_q=G.Q4_K, expert_down_q=G.Q6_K, attn_q=G.Q8_0,
                          expert_bias=False, attn_bias=False, sinks=False, qk_norm=True,
                          router_bias=False)
# small shapes with the same structure, for parity tests that the CPU oracle finishes in seconds
TINY_GPT_OSS = replace(GPT_OSS_20B, name="tiny-gpt-oss", hidden=256, layers=2, heads=8, kv_heads=2,
                       head_dim=32, experts=8, top_k=4, inter=256, vocab=1024, sliding_window=8)
TINY_QWEN3 = replace(QWEN3_30B_A3B, name="tiny-qwen3", hidden=256, layers=2, heads=4, kv_heads=2,
                     head_dim=64, experts=16, top_k=4, inter=256, vocab=1024)

# Qwen3-Coder-Next-80B shape.  Quantization of the non-expert tensors is not named by the
# benchmark: DeltaNet projections and the shared expert in Q4_K, attention in Q8_0 (stated assumption);
# rope theta is not named either (1e7 here).
QWEN3_NEXT_80B = ModelSpec(arch="qwen3next", name="Qwen3-Coder-Next-80B-synthetic", hidden=2048, layers=48,
                           heads=16, kv_heads=2, head_dim=256, experts=512, top_k=10, inter=512,
                           vocab=151936, rope_theta=1e7, eps=1e-6, sliding_window=0,
                           expert_gate_q=G.Q4_K, expert_down_q=G.Q4_K, attn_q=G.Q8_0,
                           expert_bias=False, attn_bias=False, sinks=False, qk_norm=True,
                           router_bias=False, attn_interval=4, ssm_groups=16, ssm_state=128,
                           ssm_dt_rank=32, ssm_inner=4096, ssm_conv=4, shared_inter=512, rot_factor=0.25)
TINY_QWEN3_NEXT = replace(QWEN3_NEXT_80B, name="tiny-qwen3-next", hidden=256, layers=8, experts=64,
                          inter=256, vocab=1024, ssm_groups=2, ssm_state=64, ssm_dt_rank=4, ssm_inner=512,
                          shared_inter=256)

PRESETS = {"gpt-oss-20b": GPT_OSS_20B, "gpt-oss-moe-layer": GPT_OSS_MOE_LAYER,
           "qwen3-30b-a3b": QWEN3_30B_A3B, "tiny-gpt-oss": TINY_GPT_OSS, "tiny-qwen3": TINY_QWEN3,
           "qwen3-next-80b": QWEN3_NEXT_80B, "tiny-qwen3-next": TINY_QWEN3_NEXT}


# ---- random block generators ----------------------------------------------
def tensor_rng(seed: int, name: str) -> np.random.Generator:
    h = hashlib.sha256(f"{seed}:{name}".encode()).digest()
    return np.random.default_rng(int.from_bytes(h[:8], "little"))


def _bytes(rng: np.random.Generator, n: int) -> np.ndarray:
    """n uniform bytes from the generator's raw 64-bit stream (fast path for GB-sized tensors)."""
    return rng.bit_generator.random_raw((n + 7) // 8).view(np.uint8)[:n].copy()


def rand_mxfp4(rng, n_elements: int, e_lo: int = 119, e_hi: int = 123) -> np.ndarray:
    """MXFP4 blocks: 16 bytes of uniform nibbles + e8m0 byte uniform in [e_lo, e_hi]."""
    nb = n_elements // 32
    b = _bytes(rng, nb * 17).reshape(nb, 17)
    b[:, 0] = rng.integers(e_lo, e_hi + 1, size=nb, dtype=np.uint8)
    return b.reshape(-1)


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """f32 -> Q8_0 blocks (d = amax/127 stored as f16, q = round(x/d), ggml reference rule)."""
    x = np.asarray(x, dtype=np.float32).reshape(-1, 32)
    amax = np.abs(x).max(axis=1)
    d = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        idv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    v = x * idv[:, None]
    # roundf (half away from zero): |v| <= 127, so v + 0.5*sign(v) is exact in f32
    q = np.trunc(v + np.copysign(np.float32(0.5), v)).astype(np.int8)
    out = np.empty((x.shape[0], 34), dtype=np.uint8)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(-1)


def rand_q8_0(rng, n_elements: int, std: float = 0.02) -> np.ndarray:
    return quantize_q8_0(rng.standard_normal(n_elements, dtype=np.float32) * np.float32(std))


def rand_q4_k(rng, n_elements: int, d_max: float = 1e-4, dmin_max: float = 7.5e-4) -> np.ndarray:
    """Q4_K blocks: f16 d, dmin >= 0; 12 bytes of 6-bit scales/mins (uniform 0..63); 128 nibble bytes."""
    nb = n_elements // 256
    b = _bytes(rng, nb * 144).reshape(nb, 144)
    b[:, 0:2] = (rng.random(nb, dtype=np.float32) * d_max).astype(np.float16).view(np.uint8).reshape(-1, 2)
    b[:, 2:4] = (rng.random(nb, dtype=np.float32) * dmin_max).astype(np.float16).view(np.uint8).reshape(-1, 2)
    return b.reshape(-1)


def rand_q6_k(rng, n_elements: int, d_max: float = 1.5e-5) -> np.ndarray:
    """Q6_K blocks: ql[128], qh[64] uniform; int8 scales[16] uniform over -128..127; f16 d >= 0."""
    nb = n_elements // 256
    b = _bytes(rng, nb * 210).reshape(nb, 210)
    b[:, 208:210] = (rng.random(nb, dtype=np.float32) * d_max).astype(np.float16).view(np.uint8).reshape(-1, 2)
    return b.reshape(-1)


def rand_normal_f32(rng, n: int, std: float) -> np.ndarray:
    return rng.standard_normal(n, dtype=np.float32) * np.float32(std)


_F16_NORMAL_TABLE = {}


def rand_normal_f16(rng, n: int, std: float) -> np.ndarray:
    """~N(0, std) in f16 by inverse-CDF sampling of 16-bit uniforms (fast for the 1.2 GB
    embedding / LM head tables; f16 itself is coarser than the 65536 quantile levels)."""
    tab = _F16_NORMAL_TABLE.get(std)
    if tab is None:
        from scipy.special import ndtri
        u = (np.arange(65536, dtype=np.float64) + 0.5) / 65536.0
        tab = (ndtri(u) * std).astype(np.float16)
        _F16_NORMAL_TABLE[std] = tab
    return tab[_bytes(rng, 2 * n).view(np.uint16)]


def _rand_quant(rng, qtype: int, n: int) -> np.ndarray:
    if qtype == G.MXFP4:
        return rand_mxfp4(rng, n)
    if qtype == G.Q8_0:
        return rand_q8_0(rng, n)
    if qtype == G.Q4_K:
        return rand_q4_k(rng, n)
    if qtype == G.Q6_K:
        return rand_q6_k(rng, n)
    if qtype == G.F16:
        return rand_normal_f16(rng, n, 0.02)
    if qtype == G.F32:
        return rand_normal_f32(rng, n, 0.02)
    raise ValueError(f"unsupported qtype {qtype}")


# ---- model layout ---------------------------------------------------------
TensorDef = Tuple[str, int, Tuple[int, ...], Callable[[np.random.Generator], np.ndarray]]


def tensor_defs(spec: ModelSpec) -> Iterator[TensorDef]:
    """(name, qtype, shape, generator) for every tensor of ``spec``."""
    H, E, I = spec.hidden, spec.experts, spec.inter
    ones = lambda n: (lambda rng: np.ones(n, dtype=np.float32))
    if spec.with_lm:
        yield ("token_embd.weight", spec.embed_q, (spec.vocab, H),
               lambda rng: _rand_quant(rng, spec.embed_q, spec.vocab * H))
        yield ("output_norm.weight", G.F32, (H,), ones(H))
        yield ("output.weight", spec.embed_q, (spec.vocab, H),
               lambda rng: _rand_quant(rng, spec.embed_q, spec.vocab * H))
    for L in range(spec.layers):
        p = f"blk.{L}"
        if spec.with_attention and not spec.is_attention_layer(L):
            yield (f"{p}.attn_norm.weight", G.F32, (H,), ones(H))
            yield from _deltanet_defs(spec, p)
        elif spec.with_attention:
            yield (f"{p}.attn_norm.weight", G.F32, (H,), ones(H))
            # hybrid models: the Q projection holds [Q_h, gate_h] per head (layer.rs:620-635)
            q_rows = spec.q_dim * (2 if spec.attn_interval else 1)
            for nm, rows in (("attn_q", q_rows), ("attn_k", spec.kv_dim), ("attn_v", spec.kv_dim)):
                yield (f"{p}.{nm}.weight", spec.attn_q, (rows, H),
                       (lambda r: lambda rng: _rand_quant(rng, spec.attn_q, r * H))(rows))
                if spec.attn_bias:
                    yield (f"{p}.{nm}.bias", G.F32, (rows,),
                           (lambda r: lambda rng: rand_normal_f32(rng, r, 0.01))(rows))
            yield (f"{p}.attn_output.weight", spec.attn_q, (H, spec.q_dim),
                   lambda rng: _rand_quant(rng, spec.attn_q, H * spec.q_dim))
            if spec.attn_bias:
                yield (f"{p}.attn_output.bias", G.F32, (H,), lambda rng: rand_normal_f32(rng, H, 0.01))
            if spec.sinks:
                yield (f"{p}.attn_sinks.weight", G.F32, (spec.heads,),
                       lambda rng: rand_normal_f32(rng, spec.heads, 1.0))
            if spec.qk_norm:
                yield (f"{p}.attn_q_norm.weight", G.F32, (spec.head_dim,), ones(spec.head_dim))
                yield (f"{p}.attn_k_norm.weight", G.F32, (spec.head_dim,), ones(spec.head_dim))
        norm_name = "post_attention_norm" if spec.arch == "gpt-oss" else "ffn_norm"
        yield (f"{p}.{norm_name}.weight", G.F32, (H,), ones(H))
        yield (f"{p}.ffn_gate_inp.weight", G.F32, (E, H), lambda rng: rand_normal_f32(rng, E * H, 0.02))
        if spec.router_bias:
            yield (f"{p}.ffn_gate_inp.bias", G.F32, (E,), lambda rng: rand_normal_f32(rng, E, 0.01))
        for nm, q, shp in (("ffn_gate_exps", spec.expert_gate_q, (E, I, H)),
                           ("ffn_up_exps", spec.expert_gate_q, (E, I, H)),
                           ("ffn_down_exps", spec.expert_down_q, (E, H, I))):
            yield (f"{p}.{nm}.weight", q, shp,
                   (lambda q_, n_: lambda rng: _rand_quant(rng, q_, n_))(q, int(np.prod(shp))))
            if spec.expert_bias:
                rows = shp[1]
                yield (f"{p}.{nm}.bias", G.F32, (E, rows),
                       (lambda n_: lambda rng: rand_normal_f32(rng, n_, 0.01))(E * rows))
        if spec.shared_inter:
            S, q = spec.shared_inter, spec.shared_q
            for nm, shp in (("ffn_gate_shexp", (S, H)), ("ffn_up_shexp", (S, H)), ("ffn_down_shexp", (H, S))):
                yield (f"{p}.{nm}.weight", q, shp,
                       (lambda n_: lambda rng: _rand_quant(rng, q, n_))(shp[0] * shp[1]))
            yield (f"{p}.ffn_gate_inp_shexp.weight", G.F32, (H,), lambda rng: rand_normal_f32(rng, H, 0.05))


def _deltanet_defs(spec: ModelSpec, p: str) -> Iterator[TensorDef]:
    """One Gated DeltaNet layer in the split (Unsloth) format deltanet.rs:101-137 reads: attn_qkv
    (flat Q, K, V rows), attn_gate (z), ssm_ba (flat beta, alpha rows), ssm_out, and the f32 conv1d
    [conv_dim, taps], ssm_a (= -exp(A_log)), ssm_dt.bias and ssm_norm [head_v_dim]."""
    H, nv, q = spec.hidden, spec.ssm_dt_rank, spec.ssm_q
    C, V = spec.ssm_conv_dim, spec.ssm_inner
    for nm, rows, cols in (("attn_qkv", C, H), ("attn_gate", V, H), ("ssm_ba", 2 * nv, H), ("ssm_out", H, V)):
        yield (f"{p}.{nm}.weight", q, (rows, cols), (lambda n_: lambda rng: _rand_quant(rng, q, n_))(rows * cols))
    ks = spec.ssm_conv
    yield (f"{p}.ssm_conv1d.weight", G.F32, (C, ks), lambda rng: rand_normal_f32(rng, C * ks, 0.5))
    yield (f"{p}.ssm_a", G.F32, (nv,), lambda rng: (-np.exp(rng.uniform(-1.0, 1.0, nv))).astype(np.float32))
    yield (f"{p}.ssm_dt.bias", G.F32, (nv,), lambda rng: rng.uniform(-1.0, 1.0, nv).astype(np.float32))
    hvd = V // nv
    yield (f"{p}.ssm_norm.weight", G.F32, (hvd,), lambda rng: rng.uniform(0.5, 1.5, hvd).astype(np.float32))


def metadata(spec: ModelSpec) -> Dict[str, Tuple[int, object]]:
    a = spec.arch
    m = {
        "general.architecture": (G.T_STR, a),
        "general.name": (G.T_STR, spec.name),
        "general.alignment": (G.T_U32, 32),
        f"{a}.embedding_length": (G.T_U32, spec.hidden),
        f"{a}.block_count": (G.T_U32, spec.layers),
        f"{a}.attention.head_count": (G.T_U32, spec.heads),
        f"{a}.attention.head_count_kv": (G.T_U32, spec.kv_heads),
        f"{a}.attention.key_length": (G.T_U32, spec.head_dim),
        f"{a}.expert_count": (G.T_U32, spec.experts),
        f"{a}.expert_used_count": (G.T_U32, spec.top_k),
        f"{a}.expert_feed_forward_length": (G.T_U32, spec.inter),
        f"{a}.rope.freq_base": (G.T_F32, spec.rope_theta),
        f"{a}.attention.layer_norm_rms_epsilon": (G.T_F32, spec.eps),
        f"{a}.vocab_size": (G.T_U32, spec.vocab),
    }
    if spec.sliding_window:
        m[f"{a}.attention.sliding_window"] = (G.T_U32, spec.sliding_window)
    if spec.rot_factor != 1.0:
        m[f"{a}.rope.partial_rotary_factor"] = (G.T_F32, spec.rot_factor)
    if spec.attn_interval:
        m[f"{a}.attention.full_attention_interval"] = (G.T_U32, spec.attn_interval)
        m[f"{a}.ssm.group_count"] = (G.T_U32, spec.ssm_groups)
        m[f"{a}.ssm.state_size"] = (G.T_U32, spec.ssm_state)
        m[f"{a}.ssm.time_step_rank"] = (G.T_U32, spec.ssm_dt_rank)
        m[f"{a}.ssm.inner_size"] = (G.T_U32, spec.ssm_inner)
        m[f"{a}.ssm.conv_kernel"] = (G.T_U32, spec.ssm_conv)
    return m


def build_model(spec: ModelSpec, seed: int = 0, only: Optional[Callable[[str], bool]] = None) -> G.Model:
    """Generate every tensor of ``spec`` (or those whose name passes ``only``) in memory."""
    m = G.Model()
    for k, (vt, v) in metadata(spec).items():
        m.add_meta(k, vt, v)
    for name, q, shp, gen in tensor_defs(spec):
        if only is not None and not only(name):
            continue
        m.add(name, q, shp, gen(tensor_rng(seed, name)))
    return m


def write_model(path: str, spec: ModelSpec, seed: int = 0) -> None:
    G.write_gguf(path, build_model(spec, seed))


def moe_layer_input(spec: ModelSpec, seed: int = 0) -> np.ndarray:
    """Config 0 input: hidden ~N(0,1) then RMSNorm (eps, gamma = 1)."""
    rng = tensor_rng(seed, "input.hidden")
    h = rng.standard_normal(spec.hidden, dtype=np.float32)
    ms = np.float32(np.mean(h.astype(np.float32) ** 2, dtype=np.float32))
    return (h * np.float32(1.0 / np.sqrt(ms + np.float32(spec.eps)))).astype(np.float32)


def prompt_ids(spec: ModelSpec, n: int, seed: int = 0) -> np.ndarray:
    """Prompt of ``n`` uniform random token ids."""
    return tensor_rng(seed, f"prompt.{n}").integers(0, spec.vocab, size=n, dtype=np.int64).astype(np.int32)
