"""A small Qwen3-MoE model with random weights for the decode-step tests,
and the oracle's forward_token over the same bytes (the CPU restatements of
moe.rs:1824-2073: embedding row, per layer the attention half and the MoE
block, output norm, LM head, greedy pick)."""
from dataclasses import dataclass

import numpy as np

from oracle import oracle as O

Q4_K, Q6_K, Q8_0 = 12, 14, 8


# ggml types of the model's matrices (the 30B file's mix by default)
QT_MIX = dict(embd=Q4_K, head=Q6_K, wq=Q4_K, wk=Q4_K, wv=Q6_K, wo=Q4_K, gate=Q4_K, up=Q4_K, down=Q6_K)
# config 1: every matrix q8_0; the embedding stays q4_K because the
# reference's host-side embedding dequant reads q4_K blocks only (moe.rs:1824-1833)
QT_CFG1 = dict(embd=Q4_K, head=Q8_0, wq=Q8_0, wk=Q8_0, wv=Q8_0, wo=Q8_0, gate=Q8_0, up=Q8_0, down=Q8_0)


@dataclass
class Model:
    hp: dict
    embd: np.ndarray          # qt["embd"] [n_vocab][H]
    layers: list              # dicts: attn_norm, wq.. (qtype, raw), q_norm, k_norm, ffn_norm, router, gate, up, down
    output_norm: np.ndarray
    head: np.ndarray          # qt["head"] [n_vocab][H]
    qt: dict = None           # ggml types (QT_MIX when None)

    def __post_init__(self):
        if self.qt is None:
            self.qt = dict(QT_MIX)


def make_model(seed=0, n_layers=2, H=512, n_heads=8, n_kv=2, hd=64, F=256, E=16, k=4, n_vocab=1024):
    rng = np.random.default_rng(seed)

    def q(qt, rows, cols, sigma=0.02):
        return O.quantize(qt, rng.normal(0, sigma, (rows, cols)).astype(np.float32)).reshape(-1)

    hp = dict(n_layers=n_layers, n_embd=H, n_heads=n_heads, n_kv_heads=n_kv, head_dim=hd, n_ff=F, n_expert=E,
              n_expert_used=k, n_vocab=n_vocab, rms_eps=1e-6, rope_base=1_000_000.0)
    layers = []
    for _ in range(n_layers):
        layers.append(dict(
            attn_norm=rng.uniform(0.5, 1.5, H).astype(np.float32),
            wq=(Q4_K, q(Q4_K, n_heads * hd, H)), wk=(Q4_K, q(Q4_K, n_kv * hd, H)),
            wv=(Q6_K, q(Q6_K, n_kv * hd, H)), wo=(Q4_K, q(Q4_K, H, n_heads * hd)),
            q_norm=rng.uniform(0.5, 1.5, hd).astype(np.float32), k_norm=rng.uniform(0.5, 1.5, hd).astype(np.float32),
            ffn_norm=rng.uniform(0.5, 1.5, H).astype(np.float32),
            router=rng.normal(0, 0.05, (E, H)).astype(np.float32),
            gate=q(Q4_K, E * F, H), up=q(Q4_K, E * F, H), down=q(Q6_K, E * H, F)))
    return Model(hp, q(Q4_K, n_vocab, H, 1.0), layers, rng.uniform(0.5, 1.5, H).astype(np.float32),
                 q(Q6_K, n_vocab, H, 0.05))


def make_config1(seed=1):
    """configs[0] as specified: 4 layers, hidden 512, 8 Q / 2 KV heads of 64,
    32 experts top-4, expert FFN 256, vocab 4096; every matrix q8_0 from
    N(0, 0.02) (the embedding q4_K, see QT_CFG1), router f32 N(0, 0.02),
    RMSNorm weights 1.0, eps 1e-6, RoPE theta 1e6.  Prompt: 16 ids from
    default_rng(101), 32 greedy tokens."""
    rng = np.random.default_rng(seed)
    H, nh, nkv, hd, F, E, k, nv, L = 512, 8, 2, 64, 256, 32, 4, 4096, 4
    qt = QT_CFG1

    def q(t, rows, cols):
        return O.quantize(t, rng.normal(0, 0.02, (rows, cols)).astype(np.float32)).reshape(-1)

    hp = dict(n_layers=L, n_embd=H, n_heads=nh, n_kv_heads=nkv, head_dim=hd, n_ff=F, n_expert=E,
              n_expert_used=k, n_vocab=nv, rms_eps=1e-6, rope_base=1_000_000.0)
    ones = lambda n: np.ones(n, np.float32)   # noqa: E731
    embd = q(qt["embd"], nv, H)
    layers = [dict(attn_norm=ones(H), wq=(qt["wq"], q(qt["wq"], nh * hd, H)), wk=(qt["wk"], q(qt["wk"], nkv * hd, H)),
                   wv=(qt["wv"], q(qt["wv"], nkv * hd, H)), wo=(qt["wo"], q(qt["wo"], H, nh * hd)),
                   q_norm=ones(hd), k_norm=ones(hd), ffn_norm=ones(H),
                   router=rng.normal(0, 0.02, (E, H)).astype(np.float32),
                   gate=q(qt["gate"], E * F, H), up=q(qt["up"], E * F, H), down=q(qt["down"], E * H, F))
              for _ in range(L)]
    m = Model(hp, embd, layers, ones(H), q(qt["head"], nv, H), dict(qt))
    prompt = [int(t) for t in np.random.default_rng(101).integers(0, nv, 16)]
    return m, prompt, 32


def total_cmp_argmax_last(v):
    """max_by(total_cmp) over the indices: the last index of the maximum."""
    b = np.ascontiguousarray(v, np.float32).view(np.int32).astype(np.int64)
    key = np.where(b < 0, b ^ 0x7FFFFFFF, b)
    m = key.max()
    return int(np.nonzero(key == m)[0][-1])


class OracleDecoder:
    def __init__(self, m: Model, n_ctx: int):
        self.m, self.n_ctx, self.n_past = m, n_ctx, 0
        hp = m.hp
        kvd = hp["n_kv_heads"] * hp["head_dim"]
        self.kc = [np.zeros((n_ctx, kvd), np.float32) for _ in range(hp["n_layers"])]
        self.vc = [np.zeros((n_ctx, kvd), np.float32) for _ in range(hp["n_layers"])]

    def forward_token(self, token):
        m, hp, pos = self.m, self.m.hp, self.n_past
        H = hp["n_embd"]
        rb = O.row_bytes(m.qt["embd"], H)
        x = O.dequantize(m.qt["embd"], m.embd[token * rb:(token + 1) * rb], H).reshape(-1)
        ids = []
        for li, ly in enumerate(m.layers):
            x = O.attn_block(x, ly["attn_norm"], hp["rms_eps"], hp["n_heads"], hp["n_kv_heads"], hp["head_dim"],
                             ly["q_norm"], ly["k_norm"], hp["rope_base"], [ly["wq"], ly["wk"], ly["wv"], ly["wo"]],
                             pos, self.kc[li], self.vc[li])
            r = O.moe_block(x, ly["ffn_norm"], hp["rms_eps"], ly["router"], hp["n_expert_used"], True,
                            (m.qt["gate"], m.qt["up"], m.qt["down"]), ly["gate"], ly["up"], ly["down"], hp["n_ff"])
            x = r["x"]
            ids.append(r["ids64"][:hp["n_expert_used"]])
        xn = O.rms_norm(x, m.output_norm, hp["rms_eps"])
        logits = O.matvec_q(m.qt["head"], m.head, hp["n_vocab"], H, xn)
        self.n_past += 1
        return logits, x, ids


def write_gguf(m: Model, path, arch: str = "qwen3moe", **keys) -> None:
    """The model as a qwen3moe GGUF file (styx_b200.gguf.write_decode_gguf)."""
    from styx_b200 import gguf as G
    layers = [dict(attn_norm=ly["attn_norm"], wq=ly["wq"][1], wk=ly["wk"][1], wv=ly["wv"][1], wo=ly["wo"][1],
                   q_norm=ly["q_norm"], k_norm=ly["k_norm"], ffn_norm=ly["ffn_norm"], router=ly["router"],
                   gate=ly["gate"], up=ly["up"], down=ly["down"]) for ly in m.layers]
    ly0 = m.layers[0]
    qtypes = dict(m.qt, wq=ly0["wq"][0], wk=ly0["wk"][0], wv=ly0["wv"][0], wo=ly0["wo"][0])
    G.write_decode_gguf(path, arch, m.hp, m.embd, layers, m.output_norm, m.head, qtypes, **keys)


def oracle_greedy(m: Model, prompt, n_predict, n_ctx=64):
    od = OracleDecoder(m, n_ctx)
    for t in prompt:
        lg, _, _ = od.forward_token(t)
    toks = [total_cmp_argmax_last(lg)]
    for _ in range(1, n_predict):
        lg, _, _ = od.forward_token(toks[-1])
        toks.append(total_cmp_argmax_last(lg))
    return toks
