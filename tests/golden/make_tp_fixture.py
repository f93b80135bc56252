"""Generate tests/golden/tp_decoder_logits.npz: oracle logits of a small
Llama-style decoder whose shapes split over 1, 2, 4 and 8 tensor-parallel
ranks, for the bench's and the tests' tensor-parallel parity check.

Config: vocab 1024, d_model 1024, 2 layers, 8 heads x 128 (8 KV heads),
SwiGLU 2048, Q4_0 linears, RMSNorm eps 1e-5. Weights come from
vortex_b200.decoder.synthetic_weights(seed 77) quantized by the oracle's
block quantizer (bit-identical to the product's packer); four sequences each
take an 8-token prompt (the logits after the last prompt token are stored),
then 4 teacher-forced decode steps whose tokens are stored with their
logits. The oracle is oracle/llama_oracle.py (f64, stdlib/ai/transformer.vx
block semantics).

    python tests/golden/make_tp_fixture.py
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

CFG = dict(vocab_size=1024, dim=1024, n_layers=2, n_heads=8, n_kv_heads=8, ffn_dim=2048, norm_eps=1e-5)
SEED = 77
BATCH, PROMPT, STEPS = 4, 8, 4
SEQ_IDS = [3, 10, 21, 40]
PATH = os.path.join(HERE, "tp_decoder_logits.npz")


def oracle_logits():
    from oracle import oracle as O
    from oracle.llama_oracle import LlamaOracle
    from vortex_b200.decoder import LINEAR_KEYS, synthetic_weights
    w = synthetic_weights(CFG, SEED)
    layers = []
    for l in w["layers"]:
        layers.append({k: (O.quantize_blocks(O.GGML_Q4_0, v) if k in LINEAR_KEYS else v) for k, v in l.items()})
    orc = LlamaOracle(dict(CFG), layers, O.bf16_bits_to_f32_array(w["emb_bits"]), w["final_w"], w["final_b"],
                      O.quantize_blocks(O.GGML_Q4_0, w["out"]), O.GGML_Q4_0)
    rng = np.random.default_rng(SEED + 1)
    prompts = rng.integers(0, CFG["vocab_size"], size=(BATCH, PROMPT)).astype(np.int32)
    tokens = rng.integers(0, CFG["vocab_size"], size=(STEPS, BATCH)).astype(np.int32)
    for p in range(PROMPT):
        pre = orc.step_batch(SEQ_IDS, prompts[:, p], logits=p == PROMPT - 1)
    logits = np.stack([orc.step_batch(SEQ_IDS, tokens[s]) for s in range(STEPS)])
    return dict(prompts=prompts, prefill_logits=pre.astype(np.float32), tokens=tokens,
                logits=logits.astype(np.float32), seq_ids=np.array(SEQ_IDS, dtype=np.int64),
                cfg=np.array(json.dumps(CFG)), seed=np.array(SEED))


if __name__ == "__main__":
    np.savez_compressed(PATH, **oracle_logits())
    print(PATH)
