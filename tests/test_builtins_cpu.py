"""The builtin adapters' host-side semantics (src/interpreter.rs:7278-7389,
src/kv_cache.rs:255-290): argument checks and error strings, the
QuantTensor struct the quantize builtin returns (mean _scale, quirk of
get_scale), dequantize through value_to_quant_tensor (one PerTensor scale),
compression ratios, and the batcher builtins."""
import numpy as np
import pytest

from oracle import oracle as O


def test_quantize_struct_and_errors():
    from vortex_b200 import builtins as B
    with pytest.raises(B.BuiltinError, match="quantize requires at least 3 args: data, shape, format"):
        B.quantize([1.0], [1])
    with pytest.raises(B.BuiltinError, match="quantize: unknown format 'FP3'"):
        B.quantize([1.0], [1], "FP3")
    with pytest.raises(B.BuiltinError, match="quantize: first arg must be array"):
        B.quantize(1.0, [1], "INT8")
    rng = np.random.default_rng(1)
    x = rng.standard_normal(96)
    qt = B.quantize(list(x), [8, 12], "INT8", 32)
    packed, scales, zps = O.quantize(x, O.INT8, 32)
    assert qt["_data"] == [int(b) for b in packed]
    assert qt["_scale"] == O.get_scale(scales, True)  # the mean of the group scales
    assert qt["_zero_point"] == 0 and qt["compression_ratio"] == 4.0 and qt["shape"] == [8, 12]
    # dequantize reads the struct as PerTensor with that mean scale
    want = O.dequantize(packed, 96, O.INT8, None, [qt["_scale"]], [0])
    assert B.dequantize(qt) == list(want)
    assert B.compression_ratio(B.quantize([1.0] * 64, [8, 8], "INT4")) == 8.0


def test_value_to_quant_tensor_errors():
    from vortex_b200 import builtins as B
    with pytest.raises(B.BuiltinError, match="expected QuantTensor struct"):
        B.dequantize([1, 2])
    with pytest.raises(B.BuiltinError, match="QuantTensor missing format field"):
        B.dequantize({"shape": [1], "_data": [0]})
    with pytest.raises(B.BuiltinError, match="QuantTensor missing _data"):
        B.dequantize({"format": "INT8", "shape": [1]})
    with pytest.raises(B.BuiltinError, match="dequantize requires 1 arg: qtensor"):
        B.dequantize()
    with pytest.raises(B.BuiltinError, match="quantized_matmul requires 2 args: a_q, b_q"):
        B.quantized_matmul({})


def test_batcher_builtins():
    from vortex_b200 import builtins as B
    bid = B.batcher_new(2)
    assert B.batcher_add(bid, [1, 2, 3]) == 0
    assert B.batcher_add(bid, []) == 1
    with pytest.raises(B.BuiltinError, match="batcher full"):
        B.batcher_add(bid, [4])
    assert B.batcher_active(bid) == 2
    assert B.batcher_remove(bid, 0) is True
    assert B.batcher_active(bid) == 1
    with pytest.raises(B.BuiltinError, match="invalid batcher"):
        B.batcher_active(bid + 100)
    with pytest.raises(B.BuiltinError, match="need batcher_id"):
        B.batcher_add("x", [1])
