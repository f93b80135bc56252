"""Argument checks of the single-op wrappers (vortex_b200/block_ops.py): they
reject CPU tensors, wrong dtypes and undersized outputs before any device
call, so no kernel ever sees a bad buffer. CPU only."""
import pytest

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def B():
    from vortex_b200 import block_ops
    return block_ops


def test_cpu_tensors_are_rejected(B):
    x = torch.zeros(2, 8)
    with pytest.raises(ValueError, match="CUDA tensor"):
        B.rope_embed(x, 0, 8)
    with pytest.raises(ValueError, match="CUDA tensor"):
        B.rope(x, [0.5])
    with pytest.raises(ValueError, match="CUDA tensor"):
        B.vec_add(x, x)
    with pytest.raises(ValueError, match="CUDA tensor"):
        B.swiglu(x)
    with pytest.raises(ValueError, match="CUDA tensor"):
        B.layer_norm(x, torch.ones(8), torch.zeros(8))


def test_non_tensors_are_rejected(B):
    with pytest.raises(ValueError):
        B.vec_add([1.0, 2.0], [3.0, 4.0])
