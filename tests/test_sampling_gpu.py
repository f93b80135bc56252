"""Device sampling against the oracle's literal restatement of
stdlib/ai/transformer.vx:1163-1260 (series exp, exchange sort, cutoff, LCG
draw): the sampled token must be identical for every row, including rows whose
selected probability is tied (the exchange sort's own tie order)."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _check(logits32, temperature, top_p, seeds):
    from vortex_b200 import sampling as S
    lg = torch.from_numpy(logits32).cuda()
    got = S.sample_top_p(lg, temperature, top_p, seeds).cpu().numpy()
    for r in range(logits32.shape[0]):
        want = O.sample_top_p(logits32[r].astype(np.float64), temperature, top_p, int(seeds[r]))
        assert got[r] == want, (r, got[r], want)


@pytest.mark.parametrize("vocab,temperature,top_p", [(512, 0.8, 0.9), (4096, 1.0, 0.9), (4096, 0.5, 0.5),
                                                     (1000, 2.0, 0.99), (333, 1.0, 1.0)])
def test_top_p_matches_oracle(cuda_ok, vocab, temperature, top_p):
    rng = np.random.default_rng(vocab)
    rows = 6
    logits = (rng.standard_normal((rows, vocab)) * 3).astype(np.float32)
    _check(logits, temperature, top_p, rng.integers(0, 1 << 40, rows))


def test_top_p_tied_probabilities(cuda_ok):
    """Logits on a coarse grid: most probabilities are tied, so the selected
    one usually is, and the exchange sort's tie order decides the token."""
    rng = np.random.default_rng(11)
    rows, vocab = 16, 2048
    logits = np.round(rng.standard_normal((rows, vocab)) * 2).astype(np.float32)
    _check(logits, 1.0, 0.9, np.arange(rows) * 7919 + 1)


def test_top_p_llama_vocab(cuda_ok):
    """The 7B decoder's vocabulary (32000), temperature 0.8, top_p 0.9 (the
    reference's generate settings), the generate loop's seeds 42 + t + 1."""
    rng = np.random.default_rng(32000)
    rows = 3
    logits = (rng.standard_normal((rows, 32000)) * 2).astype(np.float32)
    seeds = [43, 45, 48]
    _check(logits, 0.8, 0.9, seeds)


def test_argmax_matches_oracle(cuda_ok):
    from vortex_b200 import sampling as S
    rng = np.random.default_rng(3)
    logits = np.round(rng.standard_normal((5, 1001)), 1).astype(np.float32)
    got = S.argmax(torch.from_numpy(logits).cuda()).cpu().numpy()
    for r in range(5):
        assert got[r] == O.argmax(logits[r].astype(np.float64))
