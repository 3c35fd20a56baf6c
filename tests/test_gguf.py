"""The GGUF reader (include/styx_gguf.h) against the reference's own tests
(crates/gguf-rs/src/lib.rs:334-573, restated with the same bytes and the same
expectations), plus the writer, truncation at every byte, the UTF-8 rule and
a round trip through an independent GGUF implementation (llama.cpp's gguf
package).  CPU only: the reader is host code.
"""
import os
import struct

import numpy as np
import pytest

from styx_b200 import gguf as G


# ----------------------------------------------------------------- helpers
def u32(v):
    return struct.pack("<I", v)


def u64(v):
    return struct.pack("<Q", v)


def open_both(tmp_path, tag, data):
    """Gguf::open on a file and the in-memory parse: both must agree."""
    p = tmp_path / f"{tag}.gguf"
    p.write_bytes(data)
    results = []
    for f in (lambda: G.Gguf.open(p), lambda: G.Gguf.from_bytes(data)):
        try:
            results.append(("ok", f()))
        except G.GgufError as e:
            results.append(("err", e))
    assert results[0][0] == results[1][0], tag
    if results[0][0] == "err":
        assert (results[0][1].code, str(results[0][1])) == (results[1][1].code, str(results[1][1])), tag
    return results[0]


def assert_invalid(tmp_path, tag, data, msg_contains):
    kind, r = open_both(tmp_path, tag, data)
    assert kind == "err", f"{tag}: expected InvalidData, got Ok"
    assert r.kind == "InvalidData", f"{tag}: wrong kind {r.kind}: {r}"
    assert msg_contains in str(r), f"{tag}: message {str(r)!r} lacks {msg_contains!r}"


def header(version, tensors, kvs):
    return u32(0x46554747) + u32(version) + u64(tensors) + u64(kvs)


def kv_key(key):
    return u64(len(key)) + key.encode()


def create_test_gguf():
    """lib.rs:341-398, byte for byte."""
    b = u32(0x46554747) + u32(3) + u64(2) + u64(3)
    b += u64(12) + b"general.name" + u32(8) + u64(4) + b"test"
    b += u64(17) + b"general.alignment" + u32(4) + u32(32)
    b += u64(23) + b"tokenizer.chat_template" + u32(8) + u64(8) + b"{{chat}}"
    b += u64(2) + b"t0" + u32(2) + u64(4) + u64(2) + u32(0) + u64(0)
    b += u64(2) + b"t1" + u32(2) + u64(256) + u64(3) + u32(12) + u64(16)
    return b


# ------------------------------------------------- the reference's tests
def test_gguf_parsing(tmp_path):
    kind, g = open_both(tmp_path, "parse", create_test_gguf())
    assert kind == "ok"
    assert g.version == 3
    assert len(g.tensors) == 2
    t0, t1 = g.tensors
    assert (t0.name, t0.dims, t0.ggml_type, t0.offset, t0.size_bytes) == ("t0", [4, 2], 0, 0, 32)
    assert (t1.name, t1.dims, t1.ggml_type, t1.offset, t1.size_bytes) == ("t1", [256, 3], 12, 16, 432)
    assert g.data_start == 256      # file position after the tensor infos (228) aligned up to 32
    assert g.metadata == {"general.name": "test", "general.alignment": 32, "tokenizer.chat_template": "{{chat}}"}


def test_empty_file_is_rejected(tmp_path):
    kind, e = open_both(tmp_path, "empty", b"")
    assert kind == "err" and e.kind == "UnexpectedEof"


def test_bad_magic(tmp_path):
    b = bytearray(header(3, 0, 0))
    b[0] = ord("X")
    assert_invalid(tmp_path, "magic", bytes(b), "magic")


def test_unsupported_version(tmp_path):
    assert_invalid(tmp_path, "version", header(1, 0, 0), "version")
    assert_invalid(tmp_path, "version99", header(99, 0, 0), "version")


def test_version_2_accepted(tmp_path):
    kind, g = open_both(tmp_path, "v2", header(2, 0, 0))
    assert kind == "ok" and g.version == 2 and len(g.tensors) == 0


def test_truncated_metadata(tmp_path):
    kind, e = open_both(tmp_path, "trunc_meta", header(3, 0, 1))   # declares 1 kv, provides nothing
    assert kind == "err" and e.kind == "UnexpectedEof"


def test_string_too_long(tmp_path):
    assert_invalid(tmp_path, "longstr", header(3, 0, 1) + u64(2 ** 64 - 1), "String too long")


def test_invalid_utf8_string(tmp_path):
    b = header(3, 0, 1) + u64(4) + bytes([0xFF, 0xFE, 0xFD, 0xFC])
    assert_invalid(tmp_path, "utf8", b, "UTF-8")
    _, e = open_both(tmp_path, "utf8b", b)
    assert str(e) == "Invalid UTF-8: invalid utf-8 sequence of 1 bytes from index 0"


def test_unknown_metadata_value_type(tmp_path):
    assert_invalid(tmp_path, "valtype", header(3, 0, 1) + kv_key("k") + u32(99), "value type")


def test_array_too_long(tmp_path):
    b = header(3, 0, 1) + kv_key("k") + u32(9) + u32(4) + u64(2 ** 64 - 1)
    assert_invalid(tmp_path, "longarr", b, "Array too long")


def test_unknown_tensor_ggml_type(tmp_path):
    b = header(3, 1, 0) + kv_key("t") + u32(1) + u64(32) + u32(255) + u64(0)
    assert_invalid(tmp_path, "ggmltype", b, "type")


def test_dim_not_multiple_of_block_size(tmp_path):
    b = header(3, 1, 0) + kv_key("t") + u32(1) + u64(100) + u32(12) + u64(0)   # q4_K block is 256
    kind, e = open_both(tmp_path, "blocksize", b)
    assert kind == "err" and e.kind == "InvalidData"
    assert str(e) == "First dimension not multiple of block size"


def test_truncated_tensor_info(tmp_path):
    b = header(3, 1, 0) + kv_key("t") + u32(2)   # claims 2 dims, provides none
    kind, e = open_both(tmp_path, "trunc_tensor", b)
    assert kind == "err" and e.kind == "UnexpectedEof"


# ------------------------------------------------------------ beyond them
def test_missing_file_is_an_io_error(tmp_path):
    with pytest.raises(G.GgufError) as ei:
        G.Gguf.open(tmp_path / "absent.gguf")
    assert ei.value.kind == "Io"


def _rich_image():
    w = G.GgufWriter()
    w.add_string("general.architecture", "qwen3moe")
    w.add_u32("general.alignment", 64)
    w.add("k.u8", G.U8, 7).add("k.i8", G.I8, -7).add("k.u16", G.U16, 65000).add("k.i16", G.I16, -30000)
    w.add("k.i32", G.I32, -2 ** 31).add("k.f32", G.F32, 1.5).add("k.bool", G.BOOL, True)
    w.add("k.u64", G.U64, 2 ** 64 - 1).add("k.i64", G.I64, -2 ** 63).add("k.f64", G.F64, -0.25)
    w.add_array("k.strs", G.STRING, ["a", "", "ünïcødé"])
    w.add_array("k.f32s", G.F32, [0.5, -2.0])
    w.add_array("k.empty", 99, [])                         # unknown element type, no elements: accepted
    w.add_array("k.nested", G.ARRAY, [(G.U32, [1, 2]), (G.STRING, ["x"])])
    w.add_tensor("a", [32], 0, np.arange(32, dtype=np.float32))
    w.add_tensor("b", [256, 2], 12, np.arange(288, dtype=np.uint8))
    w.add_tensor("c", [3], 0, np.ones(3, np.float32))
    return w.to_bytes()


def test_writer_round_trip_and_value_types(tmp_path):
    data = _rich_image()
    kind, g = open_both(tmp_path, "rich", data)
    assert kind == "ok"
    m = g.metadata
    assert m["general.architecture"] == "qwen3moe" and m["general.alignment"] == 64
    assert (m["k.u8"], m["k.i8"], m["k.u16"], m["k.i16"]) == (7, -7, 65000, -30000)
    assert (m["k.i32"], m["k.f32"], m["k.bool"]) == (-2 ** 31, 1.5, True)
    assert (m["k.u64"], m["k.i64"], m["k.f64"]) == (2 ** 64 - 1, -2 ** 63, -0.25)
    assert m["k.strs"] == ["a", "", "ünïcødé"] and m["k.f32s"] == [0.5, -2.0] and m["k.empty"] == []
    assert m["k.nested"] == [[1, 2], ["x"]]
    assert g.value_types["k.u8"] == G.U8 and g.value_types["k.nested"] == G.ARRAY
    assert g.data_start % 64 == 0
    assert [t.offset for t in g.tensors] == [0, 128, 448]
    assert np.array_equal(g.tensor_data("a").view(np.float32), np.arange(32, dtype=np.float32))
    assert np.array_equal(g.tensor_data("b"), np.arange(288, dtype=np.uint8))
    assert g.get_str("general.architecture") == "qwen3moe" and g.get_u32("general.alignment") == 64
    assert g.get_f32("k.f32") == 1.5
    with pytest.raises(KeyError):
        g.get_u32("k.u64")              # present but not a u32: MoeModel::load's get_u32 refuses it
    with pytest.raises(KeyError):
        g.get_u32("no.such.key")
    g.close()


def test_every_truncation_is_rejected(tmp_path):
    data = _rich_image()
    # the key/values and tensor infos end before data_start; any cut inside
    # them fails cleanly (a cut in the data section still parses)
    g = G.Gguf.from_bytes(data)
    head = g.data_start
    g.close()
    for n in range(head - 64):
        with pytest.raises(G.GgufError) as ei:
            G.Gguf.from_bytes(data[:n])
        assert ei.value.kind == "UnexpectedEof", n


def test_data_outside_the_file_is_refused(tmp_path):
    data = _rich_image()
    cut = data[:-8]                     # the last tensor loses bytes
    g = G.Gguf.from_bytes(cut)
    assert np.array_equal(g.tensor_data("a").view(np.float32), np.arange(32, dtype=np.float32))
    with pytest.raises(G.GgufError) as ei:
        g.tensor_data("c")
    assert ei.value.kind == "InvalidData"


def test_duplicate_key_later_value_wins(tmp_path):
    b = header(3, 0, 2) + kv_key("k") + u32(4) + u32(1) + kv_key("k") + u32(8) + u64(1) + b"z"
    kind, g = open_both(tmp_path, "dup", b)
    assert kind == "ok" and g.metadata == {"k": "z"}


def test_alignment_only_from_a_u32(tmp_path):
    for vt, payload, want in ((4, u32(64), 64), (10, u64(64), 32), (5, struct.pack("<i", 64), 32)):
        b = header(3, 0, 1) + kv_key("general.alignment") + u32(vt) + payload
        kind, g = open_both(tmp_path, f"align{vt}", b)
        assert kind == "ok"
        assert g.data_start == (len(b) + want - 1) // want * want


def test_utf8_rule_matches_a_strict_decoder(tmp_path):
    """Every string verdict agrees with Python's strict UTF-8 decoder (the
    same well-formedness table); the error index and length agree too."""
    rng = np.random.default_rng(5)
    pool = [0x41, 0x7F, 0x80, 0xBF, 0xC0, 0xC1, 0xC2, 0xDF, 0xE0, 0xE1, 0xED, 0xEE, 0xEF, 0xF0, 0xF1, 0xF4,
            0xF5, 0xFF, 0x90, 0x9F, 0xA0, 0x8F]
    for trial in range(3000):
        n = int(rng.integers(0, 6))
        s = bytes(int(x) for x in rng.choice(pool, n))
        b = header(3, 0, 1) + kv_key("k") + u32(8) + u64(len(s)) + s
        try:
            s.decode("utf-8")
            ok = True
        except UnicodeDecodeError as e:
            ok = False
            incomplete = e.reason == "unexpected end of data"
            want = (f"Invalid UTF-8: incomplete utf-8 byte sequence from index {e.start}" if incomplete else
                    f"Invalid UTF-8: invalid utf-8 sequence of {e.end - e.start} bytes from index {e.start}")
        try:
            g = G.Gguf.from_bytes(b)
            assert ok, s
            assert g.metadata["k"] == s.decode("utf-8")
        except G.GgufError as err:
            assert not ok, s
            assert str(err) == want, (s, str(err), want)


def test_type_sizes():
    assert G.type_size(12) == (256, 144) and G.type_size(14) == (256, 210) and G.type_size(8) == (32, 34)
    assert G.tensor_bytes(12, [2048, 768, 128]) == 884736 * 128
    with pytest.raises(G.GgufError):
        G.type_size(4)                  # ggml type 4 (removed Q4_2) is not in the table


# --------------------------------------- an independent implementation
gguf_py = pytest.importorskip("gguf")


def test_reads_a_file_written_by_gguf_py(tmp_path):
    p = tmp_path / "by_gguf_py.gguf"
    w = gguf_py.GGUFWriter(str(p), "qwen3moe")
    w.add_uint32("qwen3moe.block_count", 2)
    w.add_float32("qwen3moe.attention.layer_norm_rms_epsilon", 1e-6)
    w.add_string("general.name", "x")
    w.add_array("tokenizer.ggml.tokens", ["a", "bb", "ccc"])
    a = np.arange(64, dtype=np.float32).reshape(2, 32)
    q = np.arange(2 * 144, dtype=np.uint8).reshape(1, 2 * 144)
    w.add_tensor("f", a)
    w.add_tensor("q", q, raw_dtype=gguf_py.GGMLQuantizationType.Q4_K)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    g = G.Gguf.open(p)
    assert g.get_str("general.architecture") == "qwen3moe"
    assert g.get_u32("qwen3moe.block_count") == 2
    assert abs(g.get_f32("qwen3moe.attention.layer_norm_rms_epsilon") - 1e-6) < 1e-12
    assert g.metadata["tokenizer.ggml.tokens"] == ["a", "bb", "ccc"]
    assert g.tensor("f").dims == [32, 2] and g.tensor("f").ggml_type == 0
    assert np.array_equal(g.tensor_data("f").view(np.float32).reshape(2, 32), a)
    assert g.tensor("q").ggml_type == 12 and g.tensor("q").dims == [512, 1]
    assert np.array_equal(g.tensor_data("q"), q.reshape(-1))


def test_gguf_py_reads_a_file_written_here(tmp_path):
    p = tmp_path / "by_styx.gguf"
    p.write_bytes(_rich_image())
    r = gguf_py.GGUFReader(str(p))
    assert r.fields["general.architecture"].contents() == "qwen3moe"
    assert r.fields["k.u64"].contents() == 2 ** 64 - 1
    assert r.fields["k.strs"].contents() == ["a", "", "ünïcødé"]
    t = {t.name: t for t in r.tensors}
    assert np.array_equal(np.asarray(t["a"].data).reshape(-1), np.arange(32, dtype=np.float32))
    assert int(t["b"].tensor_type) == 12 and list(t["b"].shape) == [256, 2]
    assert np.array_equal(np.asarray(t["b"].data).reshape(-1), np.arange(288, dtype=np.uint8))


def test_decode_model_keys_round_trip(tmp_path):
    """A whole model file (write_decode_gguf) gives back the hyper-parameters
    MoeModel::load reads (moe.rs:550-590) and every tensor it uploads."""
    from tests.decode_case import make_model, write_gguf
    m = make_model(3, n_layers=2, H=512, n_heads=8, n_kv=2, hd=128, F=256, E=8, k=2, n_vocab=300)
    path = tmp_path / "model.gguf"
    write_gguf(m, path)
    g = G.Gguf.open(path)
    hp = G.decode_params(g)
    assert (hp.n_layers, hp.n_embd, hp.n_heads, hp.n_kv_heads, hp.head_dim) == (2, 512, 8, 2, 128)
    assert (hp.n_ff, hp.n_expert, hp.n_expert_used, hp.n_vocab) == (256, 8, 2, 300)
    assert hp.qk_norm and hp.norm_topk and hp.rope_base == 1_000_000.0
    assert np.array_equal(g.tensor_data("token_embd.weight"), m.embd)
    assert np.array_equal(g.tensor_data("blk.1.attn_v.weight"), m.layers[1]["wv"][1])
    assert np.array_equal(g.tensor_data("output.weight"), m.head)
    assert g.tensor("blk.0.attn_output.weight").dims == [8 * 128, 512]
    g.close()


def test_decode_params_fallbacks(tmp_path):
    """Without attention.key_length the head size is n_embd / n_heads, without
    expert_feed_forward_length the expert width comes from ffn_gate_exps'
    dims (moe.rs:567-583); qwen2moe does not renormalise the top-k weights
    (ArchCfg.norm_topk, moe.rs:324-361)."""
    from tests.decode_case import make_model, write_gguf
    m = make_model(4, n_layers=1, H=512, n_heads=8, n_kv=2, hd=64, F=256, E=8, k=2, n_vocab=64)
    path = tmp_path / "model.gguf"
    write_gguf(m, path, arch="qwen2moe", key_length=False, ff_length=False)
    g = G.Gguf.open(path)
    assert "qwen2moe.attention.key_length" not in g.value_types
    hp = G.decode_params(g)
    assert hp.head_dim == 512 // 8 and hp.n_ff == 256 and not hp.norm_topk
    g.close()
