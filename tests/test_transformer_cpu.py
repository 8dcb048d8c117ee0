"""CPU-only checks of the transformer reference composition."""
import pytest

from silarray_b200 import transformer
from oracle import transformer_ref as TR


def test_restated_forward_matches_reference_build():
    """CPU-only: the restatement composition equals the reference build's
    block within the end-to-end tolerance (they differ only in GEMM order)."""
    import oracle as O
    if O.ref is None:
        pytest.skip("reference CPU build not present")
    cfg = transformer.Config(batch=1, seq=64, d_model=128, heads=2, d_ff=256)
    p = transformer.init_params(cfg, seed=5)
    x = transformer.init_input(cfg, seed=6)
    a = TR._restated_forward(cfg, p, x)
    b = O.ref.transformer_block(x, cfg.batch, cfg.seq, cfg.d_model, cfg.heads, cfg.d_ff, p)
    TR.check_parity(a, b, cfg)
