"""Sampling oracle pins and the continuous-batching slot table (host only).

- the oracle's series exponential (stdlib/ai/transformer.vx:36-80) agrees with
  libm to a few ulp and clamps at +-88; argmax keeps the first maximum; the
  oracle's sample_top_p returns argmax at top_p -> 0 and a token inside the
  nucleus otherwise;
- ContinuousBatcher (src/kv_cache.rs:117-154, builtins 255-290): lowest free
  slot, increasing sequence ids that are never reused, "batcher full",
  removal of a bad slot ignored, num_active.
"""
import math

import numpy as np
import pytest

from oracle import oracle as O


def test_series_exp_close_to_libm():
    for x in (0.0, -1e-9, -0.5, -1.0, -7.3, -30.0, -87.9, 0.3, 5.0):
        assert abs(O.vx_exp(x) - math.exp(x)) <= 1e-14 * math.exp(x) + 1e-300
    assert O.vx_exp(-88.5) == 0.0 and O.vx_exp(88.5) == 1.0e38


def test_argmax_first_index():
    assert O.argmax([1.0, 3.0, 3.0, 2.0]) == 1
    assert O.argmax([5.0]) == 0


def test_top_p_small_nucleus_is_argmax():
    rng = np.random.default_rng(2)
    for seed in range(5):
        l = rng.standard_normal(64)
        assert O.sample_top_p(l, 1.0, 1e-12, seed) == int(np.argmax(l))


def test_lcg_draw():
    # (1664525 * 43 + 1013904223) % 2^31 / 2^31
    assert O.lcg_uniform(43) == ((1664525 * 43 + 1013904223) % 2147483648) / 2147483648.0


def test_batcher_slots():
    from vortex_b200 import _native as N
    from vortex_b200.sampling import ContinuousBatcher, batcher_add
    b = ContinuousBatcher(3)
    assert [b.add_request([1, 2]), b.add_request([3]), b.add_request([])] == [0, 1, 2]
    assert b.num_active() == 3
    assert b.add_request([9]) is None
    with pytest.raises(N.VxbError, match="batcher full"):
        batcher_add(b, [9])
    b.remove_request(1)
    b.remove_request(17)  # ignored
    assert b.num_active() == 2
    assert b.add_request([4, 5, 6]) == 1
    s = b.slot(1)
    assert s == {"seq_id": 3, "position": 0, "is_prefill": True, "is_done": False, "n_tokens": 3}
    b.advance(1, 3)
    b.advance(1, 1, done=True)
    assert b.slot(1)["position"] == 4 and not b.slot(1)["is_prefill"] and b.slot(1)["is_done"]
    assert b.slot(0)["seq_id"] == 0 and b.slot(2)["seq_id"] == 2
