"""Seeded synthetic integer models (TEST INFRASTRUCTURE; numpy twin of the device generator).

Every tensor element is a pure function of (seed, stream, index), so the CUDA generator in
``exact_llm_b200/csrc`` produces the same integers on the device.  The recipe is integer-only
(no libm), so it is identical on every host:

    h(seed, stream, i) = mix64(mix64(seed * G + stream) + (i + 1) * G),   G = 0x9E3779B97F4A7C15
    mix64 = the splitmix64 finaliser (Steele, Lea & Flood 2014; also exact_llm.py:243-247)

    int8 "Gaussian" weight  w = clip(shr(a + b + c - 98302, 10), -127, 127)
        a, b, c = the three low 16-bit fields of h (Irwin-Hall(3): std 32)
    integer scale           M = (2^23 // isqrt(K)) + (h & 1023)          (< 2^27)
    bias (Q16)              b = (h & 0x7FFF) - 16384
    norm gain (Q16)         g = 65536 + shr(a + b + c - 98302, 2)        (std ~0.125)

Weights are (N, K) = (out, in) row-major; group scales (N, K/128) row-major.
"""
import numpy as np

from .exact_oracle import ChannelLinear, GroupLinear, OracleMoE, OracleModel, rope_tables

G64 = np.uint64(0x9E3779B97F4A7C15)
M1 = np.uint64(0xBF58476D1CE4E5B9)
M2 = np.uint64(0x94D049BB133111EB)
EMB_SHIFT = 9

# stream ids (one per tensor)
S_G1, S_G2 = 0, 1
LIN_STREAM = {"q": 2, "k": 5, "v": 8, "o": 11, "gate": 14, "up": 17, "down": 20,
              "router": 23, "sgate": 26, "sg": 29, "su": 32, "sd": 35}   # +0 weight, +1 scales, +2 bias
S_EMB, S_GF, S_HEAD_W, S_HEAD_M = 1 << 20, (1 << 20) + 1, (1 << 20) + 2, (1 << 20) + 3


def layer_stream(li, off):
    return li * 64 + off


def expert_stream(li, e, j):
    """j = 0 gate, 1 up, 2 down (each uses stream, stream+1, stream+2)."""
    return (1 << 24) + li * 4096 + e * 16 + j * 4


def mix64(z):
    with np.errstate(over="ignore"):
        z = z ^ (z >> np.uint64(30))
        z = z * M1
        z = z ^ (z >> np.uint64(27))
        z = z * M2
        return z ^ (z >> np.uint64(31))


def hashes(seed, stream, n, start=0):
    with np.errstate(over="ignore"):
        base = mix64(np.uint64(seed) * G64 + np.uint64(stream))
        idx = np.arange(start + 1, start + n + 1, dtype=np.uint64)
        return mix64(base + idx * G64)


def _tri16(h):
    f = np.uint64(0xFFFF)
    return ((h & f).astype(np.int64) + ((h >> np.uint64(16)) & f).astype(np.int64)
            + ((h >> np.uint64(32)) & f).astype(np.int64) - 98302)


def gen_weight(seed, stream, N, K):
    out = np.empty((N, K), np.int8)
    step = max(1, (1 << 24) // K)                       # bound temporaries for big matrices
    for r0 in range(0, N, step):
        r1 = min(N, r0 + step)
        v = _tri16(hashes(seed, stream, (r1 - r0) * K, r0 * K))
        out[r0:r1] = np.clip((v + 512) >> 10, -127, 127).reshape(r1 - r0, K)
    return out


def isqrt_int(n):
    r = int(n ** 0.5)
    while r * r > n:
        r -= 1
    while (r + 1) * (r + 1) <= n:
        r += 1
    return r


def gen_scale(seed, stream, n, K):
    base = (1 << 23) // isqrt_int(K)
    return base + (hashes(seed, stream, n) & np.uint64(1023)).astype(np.int64)


def gen_bias(seed, stream, n):
    return (hashes(seed, stream, n) & np.uint64(0x7FFF)).astype(np.int64) - 16384


def gen_gain(seed, stream, n):
    return 65536 + ((_tri16(hashes(seed, stream, n)) + 2) >> 2)


def group_linear(seed, stream, N, K, bias):
    w = gen_weight(seed, stream, N, K)
    M = gen_scale(seed, stream + 1, N * (K // 128), K).reshape(N, K // 128)
    b = gen_bias(seed, stream + 2, N) if bias else None
    return GroupLinear(w, M, b)


def channel_linear(seed, stream, N, K, bias):
    w = gen_weight(seed, stream, N, K)
    M = gen_scale(seed, stream + 1, N, K)
    b = gen_bias(seed, stream + 2, N) if bias else None
    return ChannelLinear(w, M, b)


# ----------------------------------------------------------------------------- configs
CONFIGS = {
    # BASELINE config 1
    "qwen2.5-0.5b": dict(D=896, H=14, KV=2, hd=64, I=4864, V=151936, NL=24, theta=1e6, tie=True, lin="group"),
    # BASELINE config 3
    "qwen2.5-7b": dict(D=3584, H=28, KV=4, hd=128, I=18944, V=152064, NL=28, theta=1e6, tie=False, lin="group"),
    # BASELINE config 5
    "qwen2.5-14b": dict(D=5120, H=40, KV=8, hd=128, I=13824, V=152064, NL=48, theta=1e6, tie=False, lin="group"),
    # BASELINE config 4 (every linear per-channel, as in experiments/moe_exact_kaggle.py:439-448)
    "qwen1.5-moe-a2.7b": dict(D=2048, H=16, KV=16, hd=128, I=1408, V=151936, NL=24, theta=1e6, tie=False,
                              lin="channel", NE=60, TOPK=4, MI=1408, SI=5632),
    # small test models
    "tiny-g128": dict(D=256, H=4, KV=2, hd=64, I=512, V=1000, NL=2, theta=1e6, tie=True, lin="group"),
    "tiny-ch": dict(D=256, H=4, KV=2, hd=64, I=384, V=777, NL=2, theta=1e4, tie=False, lin="channel"),
    "tiny-moe": dict(D=256, H=4, KV=4, hd=64, I=128, V=1000, NL=2, theta=1e6, tie=False, lin="channel",
                     NE=8, TOPK=2, MI=128, SI=256),
}


def config(name, **over):
    c = dict(CONFIGS[name])
    c.update(over)
    c.setdefault("T", 4096 + 256)
    return c


def build_model(c, seed):
    """Return an OracleModel for config dict ``c`` with weights from ``seed``."""
    D, H, KV, hd, I, V, NL = (c[k] for k in ("D", "H", "KV", "hd", "I", "V", "NL"))
    lin = group_linear if c["lin"] == "group" else channel_linear
    layers = []
    for li in range(NL):
        st = lambda nm: layer_stream(li, LIN_STREAM[nm])  # noqa: E731
        L = dict(g1=gen_gain(seed, layer_stream(li, S_G1), D), g2=gen_gain(seed, layer_stream(li, S_G2), D),
                 q=lin(seed, st("q"), H * hd, D, True), k=lin(seed, st("k"), KV * hd, D, True),
                 v=lin(seed, st("v"), KV * hd, D, True), o=lin(seed, st("o"), D, H * hd, False))
        if "NE" in c:
            L["router"] = channel_linear(seed, st("router"), c["NE"], D, False)
            L["sgate"] = channel_linear(seed, st("sgate"), 1, D, False)
            L["sg"] = channel_linear(seed, st("sg"), c["SI"], D, False)
            L["su"] = channel_linear(seed, st("su"), c["SI"], D, False)
            L["sd"] = channel_linear(seed, st("sd"), D, c["SI"], False)
            L["ex"] = [(channel_linear(seed, expert_stream(li, e, 0), c["MI"], D, False),
                        channel_linear(seed, expert_stream(li, e, 1), c["MI"], D, False),
                        channel_linear(seed, expert_stream(li, e, 2), D, c["MI"], False))
                       for e in range(c["NE"])]
        else:
            L["gate"] = lin(seed, st("gate"), I, D, False)
            L["up"] = lin(seed, st("up"), I, D, False)
            L["down"] = lin(seed, st("down"), D, I, False)
        layers.append(L)
    emb = gen_weight(seed, S_EMB, V, D)
    gf = gen_gain(seed, S_GF, D)
    head_w = emb if c["tie"] else gen_weight(seed, S_HEAD_W, V, D)
    head = ChannelLinear(head_w, gen_scale(seed, S_HEAD_M, V, D), None)
    cos, sin = rope_tables(c["T"], hd, c["theta"])

    def emb_q16(ids):
        return emb[ids].astype(np.int64) << EMB_SHIFT

    moe = OracleMoE(c["NE"], c["TOPK"]) if "NE" in c else None
    m = OracleModel(c, layers, gf, head, emb_q16, cos, sin, moe)
    m.emb_i8 = emb
    return m


def prompt_ids(seed, B, T, V):
    """Uniform prompt ids (host numpy RNG; inputs, not weights)."""
    return np.random.default_rng(seed).integers(0, V, (B, T)).astype(np.int64)


def linear_case(seed, K, N, R):
    """uniform int8 activations (as int64) and a group-128 layer."""
    x = np.random.default_rng(seed).integers(-128, 128, (R, K)).astype(np.int64)
    lin = group_linear(seed, 7, N, K, False)
    return x, lin


def float_checkpoint(c, seed):
    """Seeded float64 stand-in for a Qwen2-family checkpoint in the Hugging Face naming (conversion
    tests only): weights N(0, 0.05), norm gains 1 + N(0, 0.1), q/k/v biases N(0, 0.02)."""
    rng = np.random.default_rng(seed)
    D, I, V, qn, kn = c["D"], c["I"], c["V"], c["H"] * c["hd"], c["KV"] * c["hd"]
    t = {"model.embed_tokens.weight": rng.normal(0, 0.05, (V, D)), "model.norm.weight": 1 + rng.normal(0, 0.1, D)}
    if not c.get("tie"):
        t["lm_head.weight"] = rng.normal(0, 0.05, (V, D))
    for i in range(c["NL"]):
        p = f"model.layers.{i}."
        t[p + "input_layernorm.weight"] = 1 + rng.normal(0, 0.1, D)
        t[p + "post_attention_layernorm.weight"] = 1 + rng.normal(0, 0.1, D)
        for nm, (o, k) in {"self_attn.q_proj": (qn, D), "self_attn.k_proj": (kn, D), "self_attn.v_proj": (kn, D),
                           "self_attn.o_proj": (D, qn), "mlp.gate_proj": (I, D), "mlp.up_proj": (I, D),
                           "mlp.down_proj": (D, I)}.items():
            t[p + nm + ".weight"] = rng.normal(0, 0.05, (o, k))
            if nm in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"):
                t[p + nm + ".bias"] = rng.normal(0, 0.02, o)
    return t


CONVERT_CFG = dict(D=256, H=4, KV=2, hd=64, I=512, V=1000, NL=2, theta=1e4, tie=False, T=64)
