"""Native GGUF reader (vxb_gguf_*) against the oracle's restatement of
parse_gguf / build_gguf_bytes (src/gguf_loader.rs:341-408, 766-824) and the
reference's own GGUF tests (src/gguf_loader.rs:826-929): header fields,
metadata, tensor infos and bytes identical; errors with the reference's
messages. CPU only (no device upload)."""
import struct

import numpy as np
import pytest

from oracle import gguf_oracle as G
from oracle import oracle as O


def _file():
    rng = np.random.default_rng(3)
    w4 = O.quantize_blocks(O.GGML_Q4_0, rng.normal(0, 0.02, 3 * 64))
    w8 = O.quantize_blocks(O.GGML_Q8_0, rng.normal(0, 0.02, 2 * 96))
    f32 = rng.standard_normal(5).astype(np.float32).tobytes()
    f16 = np.arange(6, dtype=np.float16).tobytes()
    meta = [("general.architecture", G.STRING, struct.pack("<Q", 5) + b"llama"),
            ("llama.block_count", G.U32, struct.pack("<I", 42)),
            ("llama.rope.freq_base", G.F32, struct.pack("<f", 10000.0)),
            ("tokenizer.ggml.tokens", G.ARRAY, struct.pack("<IQ", G.STRING, 2) + struct.pack("<Q", 1) + b"a" +
             struct.pack("<Q", 2) + b"bc")]
    tensors = [("blk.0.attn_q.weight", [64, 3], 2, bytes(w4)), ("blk.0.ffn_down.weight", [96, 2], 8, bytes(w8)),
               ("output_norm.weight", [5], 0, f32), ("token_embd.weight", [3, 2], 1, f16)]
    return G.build_gguf_bytes(meta, tensors), tensors


def test_gguf_reader_matches_oracle_parse(tmp_path):
    from vortex_b200 import gguf
    data, tensors = _file()
    ref = G.parse_gguf(data)
    p = tmp_path / "m.gguf"
    p.write_bytes(data)
    for src in (data, str(p)):
        f = gguf.GGUFFile(src)
        assert f.version == ref["version"] == 3
        assert f.n_tensors == len(ref["tensors"]) and f.n_metadata == len(ref["metadata"])
        assert f.tensor_data_offset == ref["tensor_data_offset"] and f.alignment == 32
        for got, want, (_, _, _, blob) in zip(f.tensors(), ref["tensors"], tensors):
            assert got["name"] == want["name"] and got["type"] == want["type"]
            assert got["dims"] == want["dims"] and got["offset"] == want["offset"]
            assert got["nbytes"] == G.tensor_nbytes(want)
            assert f.tensor_bytes(got["name"]).tobytes() == blob
        assert f.meta_int("llama.block_count") == 42  # metadata U32 = 42 (reference test)
        assert f.meta_float("llama.rope.freq_base") == 10000.0
        assert f.meta_string("general.architecture") == "llama"
        f.close()


def test_gguf_reader_errors_follow_reference():
    from vortex_b200 import _native as N
    from vortex_b200 import gguf
    data, _ = _file()
    cases = [(b"XXXX" + data[4:], "invalid GGUF magic: 0x58585858 (expected 0x46475547)"),
             (data[:4] + struct.pack("<I", 1) + data[8:], "unsupported GGUF version: 1"),
             (data[:30], "unexpected EOF"),
             (b"", "unexpected EOF")]
    for blob, msg in cases:
        with pytest.raises(gguf.GGUFError) as e:
            gguf.GGUFFile(blob if blob else b"\0" * 0)
        assert msg in str(e.value), (msg, str(e.value))
        assert e.value.code == N.VXB_EFORMAT
    # unknown quant type in a tensor info
    bad = G.build_gguf_bytes([], [("t", [32], 9, b"\0" * 32)])
    with pytest.raises(gguf.GGUFError) as e:
        gguf.GGUFFile(bad)
    assert "unknown GGML quant type: 9" in str(e.value)
    with pytest.raises(gguf.GGUFError):
        gguf.GGUFFile(data).find("missing.weight")


def test_gguf_reader_version2_and_alignment():
    """A v2 header parses; general.alignment (u32) moves the data offset."""
    from vortex_b200 import gguf
    meta = [("general.alignment", G.U32, struct.pack("<I", 64))]
    blob = bytearray(G.build_gguf_bytes(meta, [("w", [32], 0, np.zeros(32, np.float32).tobytes())]))
    blob[4:8] = struct.pack("<I", 2)
    ref = G.parse_gguf(bytes(blob))
    f = gguf.GGUFFile(bytes(blob))
    assert f.version == 2 and f.alignment == 64 and f.tensor_data_offset == ref["tensor_data_offset"]
