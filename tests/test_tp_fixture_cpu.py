"""The tensor-parallel parity fixture (tests/golden/tp_decoder_logits.npz) is
the oracle's output: regenerating it gives the same arrays, and the product's
host packer turns the synthetic weights into the same Q4_0 blocks as the
oracle's quantizer (the bench loads them through the packer)."""
import json

import numpy as np

from oracle import oracle as O


def test_fixture_regenerates_identically():
    from tests.golden import make_tp_fixture as M
    stored = np.load(M.PATH)
    fresh = M.oracle_logits()
    assert json.loads(str(stored["cfg"])) == M.CFG
    for key in ("prompts", "tokens", "seq_ids"):
        assert np.array_equal(stored[key], fresh[key]), key
    for key in ("prefill_logits", "logits"):
        assert np.array_equal(stored[key], fresh[key]), key


def test_host_packer_matches_oracle_on_fixture_weights():
    from tests.golden import make_tp_fixture as M
    from vortex_b200 import quant as Q
    from vortex_b200.decoder import synthetic_weights
    w = synthetic_weights(M.CFG, M.SEED)
    for key in ("wq", "w2"):
        a = w["layers"][1][key]
        assert np.array_equal(Q.pack_blocks(Q.Q4_0, a), O.quantize_blocks(O.GGML_Q4_0, a))
    assert np.array_equal(Q.pack_blocks(Q.Q4_0, w["out"]), O.quantize_blocks(O.GGML_Q4_0, w["out"]))
