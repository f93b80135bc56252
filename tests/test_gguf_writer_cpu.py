"""GGUF writer (vortex_b200.gguf.write_gguf): files it writes parse with the
oracle's restatement of parse_gguf (src/gguf_loader.rs:341-408) and with the
native reader to the same header, metadata (types and values), tensor
descriptors and bytes; Q4_0 / Q8_0 tensors hold the oracle's block codes
(quantize_int4/int8 PerGroup 32, bit-exact); every tensor starts on an
alignment boundary, and a non-default alignment is recorded and honoured.
CPU only."""
import numpy as np
import pytest

from oracle import gguf_oracle as G
from oracle import oracle as O


def _model():
    from vortex_b200 import gguf
    rng = np.random.default_rng(11)
    w4 = rng.normal(0, 0.02, (3, 64)).astype(np.float32)
    w8 = rng.normal(0, 0.02, (2, 96)).astype(np.float32)
    norm = rng.standard_normal(5).astype(np.float32)
    emb = rng.standard_normal((2, 3)).astype(np.float32)
    raw = bytes(range(8))
    meta = {
        "general.architecture": "llama",
        "llama.block_count": 32,
        "llama.rope.freq_base": 10000.0,
        "general.big": 2**40,
        "general.flag": True,
        "tokenizer.ggml.tokens": ["a", "bc", "def"],
        "tokenizer.ggml.scores": [0.5, -1.25],
        "t.u8": gguf.GGUFValue(gguf.GGUF_U8, 200),
        "t.i8": gguf.GGUFValue(gguf.GGUF_I8, -5),
        "t.u16": gguf.GGUFValue(gguf.GGUF_U16, 60000),
        "t.i16": gguf.GGUFValue(gguf.GGUF_I16, -300),
        "t.i32": gguf.GGUFValue(gguf.GGUF_I32, -70000),
        "t.u64": gguf.GGUFValue(gguf.GGUF_U64, 2**63 + 1),
        "t.f64": gguf.GGUFValue(gguf.GGUF_F64, 1.0 / 3.0),
        "t.i32s": gguf.GGUFValue(gguf.GGUF_ARRAY, (gguf.GGUF_I32, [1, -2, 3])),
    }
    tensors = [("blk.0.attn_q.weight", w4, gguf.GGML_Q4_0), ("blk.0.ffn_down.weight", w8, gguf.GGML_Q8_0),
               ("output_norm.weight", norm, gguf.GGML_F32), ("token_embd.weight", emb, gguf.GGML_F16),
               ("raw.f32", ([2], raw), gguf.GGML_F32)]
    expect = [bytes(O.quantize_blocks(O.GGML_Q4_0, w4.astype(np.float64))),
              bytes(O.quantize_blocks(O.GGML_Q8_0, w8.astype(np.float64))), norm.tobytes(),
              emb.astype(np.float16).tobytes(), raw]
    return meta, tensors, expect


def _meta_expect():
    return {"general.architecture": (G.STRING, "llama"), "llama.block_count": (G.U32, 32),
            "llama.rope.freq_base": (G.F32, 10000.0), "general.big": (G.I64, 2**40), "general.flag": (G.BOOL, True),
            "tokenizer.ggml.tokens": (G.ARRAY, ["a", "bc", "def"]), "tokenizer.ggml.scores": (G.ARRAY, [0.5, -1.25]),
            "t.u8": (G.U8, 200), "t.i8": (G.I8, -5), "t.u16": (G.U16, 60000), "t.i16": (G.I16, -300),
            "t.i32": (G.I32, -70000), "t.u64": (G.U64, 2**63 + 1), "t.f64": (G.F64, 1.0 / 3.0),
            "t.i32s": (G.ARRAY, [1, -2, 3])}


@pytest.mark.parametrize("alignment", [32, 64, 256])
def test_written_gguf_parses_identically(tmp_path, alignment):
    from vortex_b200 import gguf
    meta, tensors, expect = _model()
    path = tmp_path / "m.gguf"
    data = gguf.write_gguf(path, meta, tensors, alignment=alignment)
    assert path.read_bytes() == data
    ref = G.parse_gguf(data)
    want_meta = _meta_expect()
    if alignment != 32:
        want_meta["general.alignment"] = (G.U32, alignment)
    assert ref["version"] == 3 and ref["metadata"] == want_meta
    assert ref["tensor_data_offset"] % alignment == 0
    f = gguf.GGUFFile(str(path))
    assert f.alignment == alignment and f.tensor_data_offset == ref["tensor_data_offset"]
    for got, want, (name, _, t), blob in zip(f.tensors(), ref["tensors"], tensors, expect):
        assert got["name"] == want["name"] == name and got["type"] == want["type"] == t
        assert got["dims"] == want["dims"] and got["offset"] == want["offset"]
        assert want["offset"] % alignment == 0
        assert f.tensor_bytes(name).tobytes() == blob
        s = ref["tensor_data_offset"] + want["offset"]
        assert data[s:s + len(blob)] == blob
    assert [t["dims"] for t in ref["tensors"]] == [[64, 3], [96, 2], [5], [3, 2], [2]]
    assert f.meta_int("llama.block_count") == 32 and f.meta_int("general.big") == 2**40
    assert f.meta_float("llama.rope.freq_base") == 10000.0
    assert f.meta_string("general.architecture") == "llama"
    f.close()


def test_writer_without_tensors_and_metadata():
    from vortex_b200 import gguf
    data = gguf.write_gguf(None)
    ref = G.parse_gguf(data)
    assert ref["version"] == 3 and ref["tensors"] == [] and ref["metadata"] == {}
    assert len(data) % 32 == 0


def test_writer_rejects_bad_input():
    from vortex_b200 import gguf
    with pytest.raises(ValueError, match="multiple of the 32-element block"):
        gguf.write_gguf(None, {}, [("w", np.zeros((2, 48), np.float32), gguf.GGML_Q4_0)])
    with pytest.raises(ValueError, match="power of two"):
        gguf.write_gguf(None, {}, [], alignment=48)
    with pytest.raises(TypeError, match="nested"):
        gguf.write_gguf(None, {"x": [[1, 2]]})
    with pytest.raises(ValueError, match="not written"):
        gguf.write_gguf(None, {}, [("w", np.zeros(32, np.float32), gguf.GGML_Q4_1)])
    with pytest.raises(ValueError, match="bytes for"):
        gguf.write_gguf(None, {}, [("w", ([3], bytes(8)), gguf.GGML_F32)])
    with pytest.raises(ValueError, match="unknown ggml type"):
        gguf.write_gguf(None, {}, [("w", ([2], bytes(8)), 24)])
