"""The GGUF parser (b2q_gguf_*) on CPU: no device is touched.

Pinned against gguf-py (GGUFWriter writes, GGUFReader reads back the same
file independently), plus files written byte by byte for what gguf-py does
not produce: versions 1 and 2, duplicate keys and tensors, and damaged
files, whose rejection mirrors GgufModelFile::open (src/inference.rs:343-446).
"""
from __future__ import annotations

import struct

import numpy as np
import pytest

import gguf_fixtures as gf


@pytest.fixture(scope="module")
def G(pkg):
    from hf_llm_b200 import gguf_file
    return gguf_file


def _lib():
    from hf_llm_b200 import _lib
    return _lib


def _tensors(seed=0):
    from hf_llm_b200 import ggml, synth
    rng = np.random.default_rng(seed)
    return [("norm", ggml.F32, [96], rng.standard_normal(96).astype(np.float32).tobytes()),
            ("w_q4k", ggml.Q4_K, [5, 512], synth.tensor_rows(ggml.Q4_K, 5, 512, seed, 1).tobytes()),
            ("w_q6k", ggml.Q6_K, [3, 256], synth.tensor_rows(ggml.Q6_K, 3, 256, seed, 2).tobytes()),
            ("w_q80", ggml.Q8_0, [7, 64], synth.tensor_rows(ggml.Q8_0, 7, 64, seed, 3).tobytes()),
            ("h16", ggml.F16, [2, 48], rng.standard_normal(96).astype(np.float16).tobytes())]


@pytest.mark.parametrize("alignment", [None, 64, 256])
def test_parser_matches_ggufpy_reader(G, tmp_path, alignment):
    import gguf
    p = tmp_path / "m.gguf"
    tensors = _tensors()
    kvs = [("t.u8", "add_uint8", 7), ("t.i8", "add_int8", -3), ("t.u16", "add_uint16", 65000),
           ("t.i16", "add_int16", -2), ("t.u32", "add_uint32", 4000000000), ("t.i32", "add_int32", -5),
           ("t.f32", "add_float32", 0.25), ("t.bool", "add_bool", True), ("t.str", "add_string", "hei på deg"),
           ("t.u64", "add_uint64", 2 ** 40), ("t.i64", "add_int64", 12), ("t.f64", "add_float64", 1.5),
           ("t.arr", "add_array", ["a", "bc", "def"]), ("t.iarr", "add_array", [1, 2, 3])]
    gf.write_ggufpy(p, "llama", kvs, tensors, alignment=alignment)
    rd = gguf.GGUFReader(str(p))
    with G.GgufFile(p) as f:
        assert f.version == 3
        keys = f.keys()
        assert keys == [k for k in rd.fields if not k.startswith("GGUF.")]  # reader's header pseudo-keys
        descs = {d.name: d for d in f.tensors()}
        assert [t.name for t in rd.tensors] == [d.name for d in f.tensors()]
        for t in rd.tensors:
            d = descs[t.name]
            assert d.dims == tuple(int(v) for v in reversed(t.shape))
            assert d.dtype == int(t.tensor_type)
            assert d.abs_offset == int(t.data_offset)
            assert d.byte_len == int(t.n_bytes)
        for name, gt, dims, data in tensors:
            assert f.tensor_bytes(name).tobytes() == data
        assert f.get_usize("t.u8") == 7 and f.get_usize("t.u16") == 65000
        assert f.get_usize("t.u32") == 4000000000 and f.get_usize("t.u64") == 2 ** 40
        assert f.get_usize("t.i64") == 12
        assert f.get_f32("t.f32") == 0.25 and f.get_f32("t.f64") == 1.5
        assert f.get_f32("t.u32") == np.float32(4000000000) and f.get_f32("t.i32") == -5.0
        assert f.get_str("t.str") == "hei på deg"
        assert f.get_str("general.architecture") == "llama"
        if alignment:
            assert f.get_usize("general.alignment") == alignment
            assert all(d.abs_offset % alignment == 0 for d in f.tensors())


def test_accessor_types_follow_ggufvalue(G, tmp_path):
    """as_usize takes u8/u16/u32/u64 and i32/i64 >= 0 only; as_f32 takes
    f32/f64/u32/i32 (src/inference.rs:203-223)."""
    L = _lib()
    p = tmp_path / "a.gguf"
    gf.write_raw(p, 3, [("neg32", gf.I32, -1), ("neg64", gf.I64, -9), ("i8", gf.I8, 5),
                        ("i16", gf.I16, 5), ("b", gf.BOOL, True), ("u16", gf.U16, 9),
                        ("f", gf.F32, 2.0), ("s", gf.STRING, "x"), ("u64", gf.U64, 3)], [])
    with G.GgufFile(p) as f:
        for k in ("neg32", "neg64", "i8", "i16", "b", "f", "s", "nope"):
            with pytest.raises(L.B2QError) as e:
                f.get_usize(k)
            assert e.value.status == L.EINVAL and "integer metadata" in str(e.value)
        assert f.get_usize("u16") == 9
        for k in ("u16", "u64", "s", "b"):
            with pytest.raises(L.B2QError):
                f.get_f32(k)
        with pytest.raises(L.B2QError):
            f.get_str("f")


@pytest.mark.parametrize("version", [1, 2, 3])
def test_versions_and_length_width(G, tmp_path, version):
    """Version 1 stores counts, lengths and dims as u32, later versions as u64."""
    p = tmp_path / f"v{version}.gguf"
    tensors = _tensors(version)
    off = gf.write_raw(p, version, [("k", gf.STRING, "v"), ("arr", gf.ARRAY, [[gf.U8, [1, 2]], [gf.U8, []]], gf.ARRAY)],
                       tensors)
    with G.GgufFile(p) as f:
        assert f.version == version
        assert f.get_str("k") == "v"
        ds = f.tensors()
        assert [d.name for d in ds] == [t[0] for t in tensors]
        assert ds[0].abs_offset == off
        for (name, gt, dims, data), d in zip(tensors, ds):
            assert d.dims == tuple(dims) and d.dtype == gt and d.byte_len == len(data)
            assert f.tensor_bytes(name).tobytes() == data


def test_duplicates_last_wins(G, tmp_path):
    """HashMap::insert semantics: a repeated key or tensor name replaces the earlier one."""
    p = tmp_path / "d.gguf"
    a, b = b"\x01" * 16, b"\x02" * 32
    gf.write_raw(p, 3, [("x", gf.U32, 1), ("y", gf.U32, 5), ("x", gf.U32, 2)],
                 [("t", 0, [4], a), ("u", 0, [2], b[:8]), ("t", 0, [8], b)])
    with G.GgufFile(p) as f:
        assert f.get_usize("x") == 2 and f.keys() == ["x", "y"]
        assert [d.name for d in f.tensors()] == ["t", "u"]
        assert f.tensor("t").dims == (8,) and f.tensor_bytes("t").tobytes() == b


def test_alignment_key_and_default(G, tmp_path):
    p = tmp_path / "al.gguf"
    off = gf.write_raw(p, 3, [("general.alignment", gf.U32, 128)], [("t", 0, [4], b"\0" * 16)], alignment=128)
    with G.GgufFile(p) as f:
        assert f.tensor("t").abs_offset == off and off % 128 == 0
    # general.alignment 0 is treated as 1 (.max(1)): data starts right after the header
    p = tmp_path / "al0.gguf"
    off = gf.write_raw(p, 3, [("general.alignment", gf.U32, 0)], [("t", 0, [4], b"\0" * 16)], alignment=1)
    with G.GgufFile(p) as f:
        assert f.tensor("t").abs_offset == off


def _expect_reject(G, path, needle):
    L = _lib()
    with pytest.raises(L.B2QError) as e:
        G.GgufFile(path)
    assert e.value.status == L.EINVAL
    assert needle in str(e.value), str(e.value)


def test_rejects_damaged_files(G, tmp_path):
    good, _ = gf.raw_bytes(3, [("a", gf.STRING, "abc"), ("b", gf.U64, 1)], _tensors())
    p = tmp_path / "x.gguf"
    p.write_bytes(b"GGUX" + good[4:])
    _expect_reject(G, p, "not a GGUF file")
    p.write_bytes(good[:4] + struct.pack("<I", 4) + good[8:])
    _expect_reject(G, p, "unsupported GGUF version 4")
    p.write_bytes(good[:4] + struct.pack("<I", 0) + good[8:])
    _expect_reject(G, p, "unsupported GGUF version 0")
    p.write_bytes(b"GGUF")
    _expect_reject(G, p, "not a GGUF file")
    # every truncation inside the header is an unexpected end; inside the data, a tensor past the end
    hdr_end = good.index(b"w_q4k") + 40
    for cut in range(16, hdr_end, 7):
        p.write_bytes(good[:cut])
        _expect_reject(G, p, "")
    p.write_bytes(good[:-1])
    _expect_reject(G, p, "extends past the end of the GGUF file")
    # a huge string length must not be trusted
    bad = bytearray(good)
    struct.pack_into("<Q", bad, 24, 2 ** 62)
    p.write_bytes(bytes(bad))
    _expect_reject(G, p, "unexpected end of GGUF file")


def test_rejects_unknown_types(G, tmp_path):
    p = tmp_path / "t.gguf"
    gf.write_raw(p, 3, [], [("t", 5, [32], b"\0" * 64)])  # GGML type 5 (removed Q4_3) is unknown
    _expect_reject(G, p, "unknown GGML type 5")
    data, _ = gf.raw_bytes(3, [("k", gf.U8, 1)], [])
    bad = bytearray(data)
    kpos = data.index(b"k") + 1
    struct.pack_into("<I", bad, kpos, 13)
    p.write_bytes(bytes(bad))
    _expect_reject(G, p, "unknown GGUF metadata value type 13")


def test_tensor_offset_past_end(G, tmp_path):
    p = tmp_path / "o.gguf"
    data, off = gf.raw_bytes(3, [], [("t", 0, [4], b"\0" * 16), ("u", 0, [4], b"\0" * 16, 4096)])
    p.write_bytes(data[:off + 4096 + 15])  # u's last byte is cut off
    _expect_reject(G, p, "tensor 'u' extends past the end")


def test_llama_config_keys_and_defaults(G, tmp_path, pkg):
    from hf_llm_b200 import ggml, synth
    cfg = dict(n_layers=3, n_embd=256, n_heads=4, n_kv_heads=2, head_dim=64, n_ff=512, n_vocab=300,
               rms_eps=1e-6, rope_theta=500000.0)
    tok = ("token_embd.weight", ggml.Q4_K, [300, 256], synth.tensor_rows(ggml.Q4_K, 300, 256, 1, 1).tobytes())
    gate = ("blk.0.ffn_gate.weight", ggml.Q4_K, [512, 256], synth.tensor_rows(ggml.Q4_K, 512, 256, 1, 2).tobytes())
    p = tmp_path / "c.gguf"
    gf.write_ggufpy(p, "qwen2", gf.llama_kvs(cfg, "qwen2"), [tok, gate])
    with G.GgufFile(p) as f:
        got = f.llama_config("qwen2")
        assert got == pytest.approx(cfg)
        # arch without keys falls back to "llama.", which this file lacks
        L = _lib()
        with pytest.raises(L.B2QError) as e:
            f.llama_config("mistral")
        assert "llama.block_count" in str(e.value)
    # only the required keys: head_count_kv = head_count, key_length = n_embd / n_heads,
    # eps 1e-5, freq_base 10000
    p = tmp_path / "d.gguf"
    gf.write_ggufpy(p, "llama", [("llama.block_count", "add_uint32", 3),
                                 ("llama.embedding_length", "add_uint32", 256),
                                 ("llama.attention.head_count", "add_uint32", 4)], [tok, gate])
    with G.GgufFile(p) as f:
        got = f.llama_config()
        assert got == pytest.approx(dict(n_layers=3, n_embd=256, n_heads=4, n_kv_heads=4, head_dim=64,
                                         n_ff=512, n_vocab=300, rms_eps=1e-5, rope_theta=10000.0))

