"""Transformer block forward on the GPU vs the reference CPU build of the same
graph (oracle/_ref: every op a sil:: array op on Device::CPU), end-to-end
tolerance |g - r| <= 2e-4 (1 + |r|)."""
import numpy as np
import pytest
import torch

from silarray_b200 import gpu, transformer

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cfg", [transformer.Config(batch=2, seq=128, d_model=256, heads=4, d_ff=1024),
                                 transformer.Config(batch=1, seq=200, d_model=192, heads=3, d_ff=500),
                                 transformer.Config(batch=2, seq=512, d_model=768, heads=12, d_ff=3072)],
                         ids=["small", "ragged", "bench-shape-2seq"])
def test_block_forward(cuda, cfg):
    p = transformer.init_params(cfg, seed=3)
    x = transformer.init_input(cfg, seed=4)
    blk = transformer.Block(cfg, p, device="cuda")
    out = blk.forward(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    ref = transformer.reference_forward(cfg, p, x)
    transformer.check_parity(out.cpu().numpy(), ref, cfg)
    gpu.device_status()
