"""GGUF files: the reader (through include/styx_gguf.h), a writer, and the
MoE-block loader.

`Gguf` mirrors gguf_rs::Gguf (crates/gguf-rs/src/lib.rs:33-38): `version`,
`metadata` (key -> value), `tensors` (TensorInfo list) and `data_start`; the
parse itself is the library's C++ restatement of Gguf::open, with the file
memory-mapped so `tensor_data` views a tensor's bytes in place.

`GgufWriter` writes the same container (header, key/values, tensor infos,
data aligned to general.alignment or 32), which is how the synthetic model
files of the benchmark configurations are produced.

`load_moe_layers` builds the MoE block's per-layer weights from a model file
the way MoeModel::load reads them (crates/model/src/moe.rs:538-599,
856-892, 1056-1078): the architecture's metadata keys, ffn_norm (or
post_attention_norm), the f32 router ffn_gate_inp and the three expert
tensors ffn_{gate,up,down}_exps, each one buffer of n_expert contiguous slabs.
`load_decode_model` adds the rest of MoeModel::load (moe.rs:996-1108): the
embedding, the attention tensors and norms of every layer, output_norm and
the LM head, into a `styx_b200.decode.DecodeModel`.
"""
from __future__ import annotations

import ctypes as C
import struct
from dataclasses import dataclass
from typing import Any, Iterable, Optional, Sequence

import numpy as np

from . import _lib
from ._lib import lib

U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<?",
        U64: "<Q", I64: "<q", F64: "<d"}
MAGIC = 0x46554747

# ArchCfg.norm_topk per supported architecture (moe.rs:324-361)
NORM_TOPK = {"qwen3moe": True, "olmoe": False, "qwen2moe": False, "qwen3next": True}


class GgufError(Exception):
    """A rejected file.  `kind` names the reference's io::ErrorKind:
    "InvalidData", "UnexpectedEof", or "Io" for open / mapping failures."""
    KINDS = {_lib.STYX_EDATA: "InvalidData", _lib.STYX_EEOF: "UnexpectedEof", _lib.STYX_EIO: "Io",
             _lib.STYX_ENOMEM: "OutOfMemory", _lib.STYX_EINVAL: "InvalidInput"}

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code
        self.kind = self.KINDS.get(code, "Other")
        self.message = message


def _check(rc: int) -> None:
    if rc != _lib.STYX_OK:
        m = lib().styx_last_error()
        raise GgufError(rc, m.decode() if m else "")


@dataclass
class TensorInfo:
    """gguf_rs::TensorInfo (lib.rs:23-30)."""
    name: str
    dims: list
    ggml_type: int
    offset: int
    size_bytes: int


class Gguf:
    """A parsed GGUF file (gguf_rs::Gguf)."""

    def __init__(self, handle: int, keep: Any = None):
        self._h = C.c_void_p(handle)
        self._keep = keep            # the caller's buffer for from_bytes
        self._close = lib().styx_gguf_close
        L = lib()
        self.version = int(L.styx_gguf_version(self._h))
        self.data_start = int(L.styx_gguf_data_start(self._h))
        self.file_bytes = int(L.styx_gguf_file_bytes(self._h))
        self.metadata: dict = {}
        self.value_types: dict = {}
        for i in range(L.styx_gguf_kv_count(self._h)):
            key = C.c_char_p()
            node = C.c_uint64()
            _check(L.styx_gguf_kv_key(self._h, i, C.byref(key)))
            _check(L.styx_gguf_kv_value(self._h, i, C.byref(node)))
            k = key.value.decode()
            self.metadata[k] = self._node(node.value)
            vt = C.c_uint32()
            _check(L.styx_gguf_node_type(self._h, node.value, C.byref(vt), None, None))
            self.value_types[k] = int(vt.value)
        self.tensors: list = []
        info = _lib.GgufTensorInfo()
        for i in range(L.styx_gguf_tensor_count(self._h)):
            _check(L.styx_gguf_tensor(self._h, i, C.byref(info)))
            self.tensors.append(TensorInfo(info.name.decode(), [int(info.dims[d]) for d in range(info.n_dims)],
                                           int(info.ggml_type), int(info.offset), int(info.size_bytes)))
        self._index = {}
        for i, t in enumerate(self.tensors):
            self._index.setdefault(t.name, i)

    # ---------------------------------------------------------------- open
    @classmethod
    def open(cls, path) -> "Gguf":
        """Gguf::open (lib.rs:41-120)."""
        h = C.c_void_p()
        _check(lib().styx_gguf_open(str(path).encode(), C.byref(h)))
        return cls(h.value)

    @classmethod
    def from_bytes(cls, data: bytes) -> "Gguf":
        """The same parse over an in-memory image (kept alive by the object)."""
        buf = C.create_string_buffer(bytes(data), len(data)) if len(data) else None
        h = C.c_void_p()
        _check(lib().styx_gguf_open_memory(buf, len(data), C.byref(h)))
        return cls(h.value, keep=buf)

    def close(self) -> None:
        if self._h:
            self._close(self._h)
            self._h = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---------------------------------------------------------------- values
    def _node(self, node: int):
        L = lib()
        vt, et, n = C.c_uint32(), C.c_uint32(), C.c_uint64()
        _check(L.styx_gguf_node_type(self._h, node, C.byref(vt), C.byref(et), C.byref(n)))
        vt, et, n = int(vt.value), int(et.value), int(n.value)
        if vt == STRING:
            return self._string(node, 0)
        if vt != ARRAY:
            return self._scalar(node, 0, vt)
        if n == 0:
            return []
        if et == STRING:
            return [self._string(node, i) for i in range(n)]
        if et == ARRAY:
            out = []
            for i in range(n):
                e = C.c_uint64()
                _check(L.styx_gguf_node_elem(self._h, node, i, C.byref(e)))
                out.append(self._node(e.value))
            return out
        return [self._scalar(node, i, et) for i in range(n)]

    def _scalar(self, node: int, index: int, vt: int):
        buf = (C.c_uint8 * 8)()
        _check(lib().styx_gguf_node_scalar(self._h, node, index, buf))
        fmt = _FMT[vt]
        return struct.unpack(fmt, bytes(buf)[: struct.calcsize(fmt)])[0]

    def _string(self, node: int, index: int) -> str:
        s, n = C.c_void_p(), C.c_uint64()
        _check(lib().styx_gguf_node_string(self._h, node, index, C.byref(s), C.byref(n)))
        return C.string_at(s.value, n.value).decode() if n.value else ""

    def get_u32(self, key: str) -> int:
        """MoeModel::load's get_u32 (moe.rs:538-543): present and a u32."""
        v = C.c_uint32()
        rc = lib().styx_gguf_get_u32(self._h, key.encode(), C.byref(v))
        if rc != _lib.STYX_OK:
            raise KeyError(f"missing/unexpected {key}: {self.metadata.get(key)!r}")
        return int(v.value)

    def get_f32(self, key: str) -> float:
        """MoeModel::load's get_f32 (moe.rs:544-549): present and an f32."""
        v = C.c_float()
        rc = lib().styx_gguf_get_f32(self._h, key.encode(), C.byref(v))
        if rc != _lib.STYX_OK:
            raise KeyError(f"missing/unexpected {key}: {self.metadata.get(key)!r}")
        return float(v.value)

    def get_str(self, key: str) -> str:
        s, n = C.c_void_p(), C.c_uint64()
        rc = lib().styx_gguf_get_str(self._h, key.encode(), C.byref(s), C.byref(n))
        if rc != _lib.STYX_OK:
            raise KeyError(f"missing/unexpected {key}: {self.metadata.get(key)!r}")
        return C.string_at(s.value, n.value).decode() if n.value else ""

    # ---------------------------------------------------------------- tensors
    def tensor(self, name: str) -> TensorInfo:
        return self.tensors[self._index[name]]

    def has_tensor(self, name: str) -> bool:
        return name in self._index

    def tensor_data(self, name: str) -> np.ndarray:
        """The tensor's bytes in place (uint8, read-only view valid while the
        file is open); refused if they do not lie inside the file."""
        i = self._index[name]
        p = C.c_void_p()
        _check(lib().styx_gguf_tensor_data(self._h, i, C.byref(p)))
        n = self.tensors[i].size_bytes
        if n == 0:
            return np.zeros(0, np.uint8)
        arr = np.ctypeslib.as_array((C.c_uint8 * n).from_address(p.value))
        arr.flags.writeable = False
        return arr


def type_size(ggml_type: int) -> tuple:
    """(elements, bytes) per block of a ggml type (compute_size_bytes)."""
    be, bb = C.c_uint64(), C.c_uint64()
    _check(lib().styx_gguf_type_size(ggml_type, C.byref(be), C.byref(bb)))
    return int(be.value), int(bb.value)


def tensor_bytes(ggml_type: int, dims: Sequence[int]) -> int:
    arr = (C.c_uint64 * max(len(dims), 1))(*dims)
    out = C.c_uint64()
    _check(lib().styx_gguf_tensor_bytes(ggml_type, arr, len(dims), C.byref(out)))
    return int(out.value)


# ---------------------------------------------------------------- writer
class GgufWriter:
    """Builds a GGUF image: header, key/values in insertion order, tensor
    infos, then the tensor data, each tensor at an offset that is a multiple
    of the alignment (general.alignment when set as a u32, else 32), the
    data section starting at the same rounded-up position the reader
    computes."""

    def __init__(self, version: int = 3):
        self.version = version
        self.kvs: list = []
        self.tensors: list = []

    def add(self, key: str, vtype: int, value, elem_type: Optional[int] = None) -> "GgufWriter":
        self.kvs.append((key, vtype, value, elem_type))
        return self

    def add_u32(self, key, v):
        return self.add(key, U32, int(v))

    def add_f32(self, key, v):
        return self.add(key, F32, float(v))

    def add_string(self, key, v):
        return self.add(key, STRING, str(v))

    def add_array(self, key, elem_type, values):
        return self.add(key, ARRAY, list(values), elem_type)

    def add_tensor(self, name: str, dims: Sequence[int], ggml_type: int, data) -> "GgufWriter":
        raw = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        need = tensor_bytes(ggml_type, dims)
        if raw.size != need:
            raise ValueError(f"{name}: {raw.size} bytes for {need} ({list(dims)}, type {ggml_type})")
        self.tensors.append((name, [int(d) for d in dims], int(ggml_type), raw))
        return self

    def _alignment(self) -> int:
        a = 32
        for key, vt, v, _ in self.kvs:
            if key == "general.alignment":
                a = int(v) if vt == U32 else 32   # the last one wins, as in the reader
        return a

    @staticmethod
    def _str(s: str) -> bytes:
        b = s.encode()
        return struct.pack("<Q", len(b)) + b

    def _value(self, vt: int, v, et: Optional[int]) -> bytes:
        if vt in _FMT:
            return struct.pack(_FMT[vt], v)
        if vt == STRING:
            return self._str(v)
        if vt == ARRAY:
            if et is None:
                raise ValueError("array element type missing")
            out = struct.pack("<IQ", et, len(v))
            for x in v:
                if et == ARRAY:
                    inner_et, inner = x
                    out += self._value(ARRAY, inner, inner_et)
                else:
                    out += self._value(et, x, None)
            return out
        raise ValueError(f"value type {vt}")

    def to_bytes(self) -> bytes:
        a = self._alignment()
        head = struct.pack("<IIQQ", MAGIC, self.version, len(self.tensors), len(self.kvs))
        for key, vt, v, et in self.kvs:
            head += self._str(key) + struct.pack("<I", vt) + self._value(vt, v, et)
        offsets, off = [], 0
        for _, _, _, raw in self.tensors:
            off = (off + a - 1) // a * a
            offsets.append(off)
            off += raw.size
        for (name, dims, t, _), o in zip(self.tensors, offsets):
            head += self._str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
            head += struct.pack("<IQ", t, o)
        data_start = (len(head) + a - 1) // a * a
        out = bytearray(head)
        out += b"\0" * (data_start - len(head))
        for (_, _, _, raw), o in zip(self.tensors, offsets):
            out += b"\0" * (data_start + o - len(out))
            out += raw.tobytes()
        return bytes(out)

    def write(self, path) -> None:
        with open(path, "wb") as f:
            f.write(self.to_bytes())


# ---------------------------------------------------------------- MoE layers
def moe_dims(g: Gguf):
    """(arch, n_layers, ops.Dims) from a model file's metadata, as
    MoeModel::load reads them (moe.rs:550-586)."""
    from . import ops
    arch = g.get_str("general.architecture")
    if arch not in NORM_TOPK:
        raise ValueError(f"unsupported architecture {arch!r}")
    n_layers = g.get_u32(f"{arch}.block_count")
    n_embd = g.get_u32(f"{arch}.embedding_length")
    n_expert = g.get_u32(f"{arch}.expert_count")
    n_used = g.get_u32(f"{arch}.expert_used_count")
    key = f"{arch}.expert_feed_forward_length"
    if g.value_types.get(key) == U32:
        n_ff = g.get_u32(key)
    elif g.has_tensor("blk.0.ffn_gate_exps.weight"):
        n_ff = g.tensor("blk.0.ffn_gate_exps.weight").dims[1]
    else:
        raise ValueError("no expert_feed_forward_length key and no ffn_gate_exps tensor")
    eps = g.get_f32(f"{arch}.attention.layer_norm_rms_epsilon")
    if n_used > _lib.IDS_PER_LAYER // 4:
        raise ValueError("the top-k is capped at 16 (moe.rs:587)")
    return arch, n_layers, ops.Dims(n_embd, n_ff, n_expert, n_used, NORM_TOPK[arch], eps)


def load_moe_layers(g: Gguf, device: int = 0, layers: Optional[Iterable[int]] = None,
                    experts_in_host: bool = False):
    """The MoE block's LayerWeights for `layers` (all by default): ffn_norm
    (or post_attention_norm) and the f32 router on the device; the expert
    tensors on the device, or in pinned host memory (the GTT tier) when
    experts_in_host.  Returns (dims, [LayerWeights], host buffers to keep)."""
    import torch

    from . import ops
    _, n_layers, dims = moe_dims(g)
    dev = f"cuda:{device}"
    E, H, F = dims.n_expert, dims.n_embd, dims.n_ff
    out, keep = [], []

    def f32(name, shape):
        t = g.tensor(name)
        if t.ggml_type != _lib.F32:
            raise ValueError(f"{name} not f32")
        a = g.tensor_data(name).view(np.float32).reshape(shape)
        return torch.from_numpy(a.copy()).to(dev)

    def experts(name, rows, cols):
        t = g.tensor(name)
        if t.ggml_type not in _lib.BLOCK:
            raise ValueError(f"{name}: ggml type {t.ggml_type} is not an expert format of the block")
        if t.dims != [cols, rows, E]:
            raise ValueError(f"{name}: dims {t.dims}, expected {[cols, rows, E]}")
        raw = g.tensor_data(name)
        if experts_in_host:
            hb = ops.HostBuffer(raw.size, device)
            hb.tensor.copy_(torch.from_numpy(raw.copy()))
            keep.append(hb)
            full = hb.tensor
        else:
            full = torch.from_numpy(raw.copy()).to(dev)
        return ops.Experts(t.ggml_type, full, t.size_bytes // E)

    for l in (range(n_layers) if layers is None else layers):
        norm = f"blk.{l}.ffn_norm.weight"
        if not g.has_tensor(norm):
            norm = f"blk.{l}.post_attention_norm.weight"
        router = g.tensor(f"blk.{l}.ffn_gate_inp.weight")
        if router.dims != [H, E]:
            raise ValueError(f"ffn_gate_inp dims {router.dims}, expected {[H, E]}")
        out.append(ops.LayerWeights(
            ffn_norm=f32(norm, (H,)), router=f32(f"blk.{l}.ffn_gate_inp.weight", (E, H)),
            gate=experts(f"blk.{l}.ffn_gate_exps.weight", F, H),
            up=experts(f"blk.{l}.ffn_up_exps.weight", F, H),
            down=experts(f"blk.{l}.ffn_down_exps.weight", H, F)))
    return dims, out, keep


def write_moe_gguf(path, arch: str, n_embd: int, n_ff: int, n_expert: int, n_expert_used: int, rms_eps: float,
                   layers: Sequence[dict], alignment: Optional[int] = None) -> None:
    """A model file holding only what the MoE block reads: the architecture
    keys and, per layer, ffn_norm (f32 [H]), ffn_gate_inp (f32, dims [H, E]),
    ffn_gate_exps / ffn_up_exps (dims [H, F, E]) and ffn_down_exps
    (dims [F, H, E]).  Each layer dict holds numpy arrays: norm, router
    (E x H), gate, up, down (the raw expert bytes) and qtypes (gate, up, down)."""
    w = GgufWriter()
    w.add_string("general.architecture", arch)
    if alignment is not None:
        w.add_u32("general.alignment", alignment)
    w.add_u32(f"{arch}.block_count", len(layers))
    w.add_u32(f"{arch}.embedding_length", n_embd)
    w.add_u32(f"{arch}.expert_count", n_expert)
    w.add_u32(f"{arch}.expert_used_count", n_expert_used)
    w.add_u32(f"{arch}.expert_feed_forward_length", n_ff)
    w.add_f32(f"{arch}.attention.layer_norm_rms_epsilon", rms_eps)
    for l, ly in enumerate(layers):
        qg, qu, qd = ly["qtypes"]
        w.add_tensor(f"blk.{l}.ffn_norm.weight", [n_embd], _lib.F32, np.asarray(ly["norm"], np.float32))
        w.add_tensor(f"blk.{l}.ffn_gate_inp.weight", [n_embd, n_expert], _lib.F32,
                     np.asarray(ly["router"], np.float32))
        w.add_tensor(f"blk.{l}.ffn_gate_exps.weight", [n_embd, n_ff, n_expert], qg, ly["gate"])
        w.add_tensor(f"blk.{l}.ffn_up_exps.weight", [n_embd, n_ff, n_expert], qu, ly["up"])
        w.add_tensor(f"blk.{l}.ffn_down_exps.weight", [n_ff, n_embd, n_expert], qd, ly["down"])
    w.write(path)


# ------------------------------------------------------------ the whole decode model
def decode_params(g: Gguf):
    """DecodeParams from a model file's metadata (MoeModel::load,
    moe.rs:550-590): the MoE keys, attention.head_count / head_count_kv,
    attention.key_length (else n_embd / n_heads), rope.freq_base, and
    n_vocab from token_embd's dims."""
    from .decode import DecodeParams
    arch, n_layers, dims = moe_dims(g)
    n_heads = g.get_u32(f"{arch}.attention.head_count")
    n_kv = g.get_u32(f"{arch}.attention.head_count_kv")
    key = f"{arch}.attention.key_length"
    head_dim = g.get_u32(key) if g.value_types.get(key) == U32 else dims.n_embd // n_heads
    rope_base = g.get_f32(f"{arch}.rope.freq_base")
    n_vocab = g.tensor("token_embd.weight").dims[1]
    return DecodeParams(n_layers, dims.n_embd, n_heads, n_kv, head_dim, dims.n_ff, dims.n_expert,
                        dims.n_expert_used, n_vocab, dims.rms_eps, rope_base, dims.norm_topk,
                        g.has_tensor("blk.0.attn_q_norm.weight"))


def load_decode_model(g: Gguf, n_ctx: int, device: int = 0, experts_in_host: bool = False, kv_page: int = 0):
    """A DecodeModel (styx_b200.decode) from a model file, as MoeModel::load
    uploads it (moe.rs:996-1108): token_embd (the embedding rows), per layer
    attn_norm, attn_q / attn_k / attn_v / attn_output, attn_q_norm /
    attn_k_norm when present and the MoE block's tensors, then output_norm
    and output (the LM head).  kv_page > 0 grows the KV caches page by page
    up to n_ctx (moe.rs:1802-1822).  Returns (model, host buffers to keep)."""
    import torch

    from . import ops
    from .decode import DecodeLayer, DecodeModel
    hp = decode_params(g)
    dev = f"cuda:{device}"
    H, qd, kvd = hp.n_embd, hp.n_heads * hp.head_dim, hp.n_kv_heads * hp.head_dim

    def f32(name, n):
        t = g.tensor(name)
        if t.ggml_type != _lib.F32 or t.dims != [n]:
            raise ValueError(f"{name}: f32 [{n}] expected, got type {t.ggml_type} dims {t.dims}")
        return torch.from_numpy(g.tensor_data(name).view(np.float32).copy()).to(dev)

    def dense(name, rows, cols):
        t = g.tensor(name)
        if t.ggml_type not in _lib.BLOCK:
            raise ValueError(f"{name}: ggml type {t.ggml_type} is not a supported block format")
        if t.dims != [cols, rows]:
            raise ValueError(f"{name}: dims {t.dims}, expected {[cols, rows]}")
        return ops.DenseWeight(t.ggml_type, torch.from_numpy(g.tensor_data(name).copy()).to(dev))

    _, moe_layers, keep = load_moe_layers(g, device, experts_in_host=experts_in_host)
    layers = []
    for l, moe in enumerate(moe_layers):
        n = lambda s: f"blk.{l}.{s}.weight"   # noqa: E731
        attn = ops.AttnWeights(f32(n("attn_norm"), H), dense(n("attn_q"), qd, H), dense(n("attn_k"), kvd, H),
                               dense(n("attn_v"), kvd, H), dense(n("attn_output"), H, qd),
                               q_norm=f32(n("attn_q_norm"), hp.head_dim) if hp.qk_norm else None,
                               k_norm=f32(n("attn_k_norm"), hp.head_dim) if hp.qk_norm else None)
        layers.append(DecodeLayer(attn, moe))
    model = DecodeModel(hp, dense("token_embd.weight", hp.n_vocab, H), layers, f32("output_norm.weight", H),
                        dense("output.weight", hp.n_vocab, H), n_ctx, device, kv_page=kv_page)
    return model, keep


def write_decode_gguf(path, arch: str, hp: dict, embd, layers: Sequence[dict], output_norm, head,
                      qtypes: dict, key_length: bool = True, ff_length: bool = True) -> None:
    """A whole Qwen3-MoE model file: the keys decode_params reads and the
    tensors load_decode_model uploads.  hp: n_layers, n_embd, n_heads,
    n_kv_heads, head_dim, n_ff, n_expert, n_expert_used, n_vocab, rms_eps,
    rope_base.  layers: dicts of numpy arrays (attn_norm, wq, wk, wv, wo raw
    bytes, q_norm, k_norm or None, ffn_norm, router, gate, up, down raw
    bytes); qtypes: the ggml types of embd, head, wq, wk, wv, wo, gate, up,
    down.  key_length / ff_length False leave out attention.key_length and
    expert_feed_forward_length, as files of architectures whose head size is
    n_embd / n_heads and whose expert width is read from ffn_gate_exps do
    (olmoe, qwen2moe; moe.rs:567-583)."""
    H, E, F = hp["n_embd"], hp["n_expert"], hp["n_ff"]
    qd, kvd = hp["n_heads"] * hp["head_dim"], hp["n_kv_heads"] * hp["head_dim"]
    w = GgufWriter()
    w.add_string("general.architecture", arch)
    w.add_u32(f"{arch}.block_count", len(layers))
    w.add_u32(f"{arch}.embedding_length", H)
    w.add_u32(f"{arch}.attention.head_count", hp["n_heads"])
    w.add_u32(f"{arch}.attention.head_count_kv", hp["n_kv_heads"])
    if key_length:
        w.add_u32(f"{arch}.attention.key_length", hp["head_dim"])
    w.add_u32(f"{arch}.expert_count", E)
    w.add_u32(f"{arch}.expert_used_count", hp["n_expert_used"])
    if ff_length:
        w.add_u32(f"{arch}.expert_feed_forward_length", F)
    w.add_f32(f"{arch}.attention.layer_norm_rms_epsilon", hp["rms_eps"])
    w.add_f32(f"{arch}.rope.freq_base", hp["rope_base"])
    w.add_tensor("token_embd.weight", [H, hp["n_vocab"]], qtypes["embd"], embd)
    for l, ly in enumerate(layers):
        n = lambda s: f"blk.{l}.{s}.weight"   # noqa: E731
        w.add_tensor(n("attn_norm"), [H], _lib.F32, np.asarray(ly["attn_norm"], np.float32))
        w.add_tensor(n("attn_q"), [H, qd], qtypes["wq"], ly["wq"])
        w.add_tensor(n("attn_k"), [H, kvd], qtypes["wk"], ly["wk"])
        w.add_tensor(n("attn_v"), [H, kvd], qtypes["wv"], ly["wv"])
        w.add_tensor(n("attn_output"), [qd, H], qtypes["wo"], ly["wo"])
        if ly.get("q_norm") is not None:
            w.add_tensor(n("attn_q_norm"), [hp["head_dim"]], _lib.F32, np.asarray(ly["q_norm"], np.float32))
            w.add_tensor(n("attn_k_norm"), [hp["head_dim"]], _lib.F32, np.asarray(ly["k_norm"], np.float32))
        w.add_tensor(n("ffn_norm"), [H], _lib.F32, np.asarray(ly["ffn_norm"], np.float32))
        w.add_tensor(n("ffn_gate_inp"), [H, E], _lib.F32, np.asarray(ly["router"], np.float32))
        w.add_tensor(n("ffn_gate_exps"), [H, F, E], qtypes["gate"], ly["gate"])
        w.add_tensor(n("ffn_up_exps"), [H, F, E], qtypes["up"], ly["up"])
        w.add_tensor(n("ffn_down_exps"), [F, H, E], qtypes["down"], ly["down"])
    w.add_tensor("output_norm.weight", [H], _lib.F32, np.asarray(output_norm, np.float32))
    w.add_tensor("output.weight", [H, hp["n_vocab"]], qtypes["head"], head)
    w.write(path)
