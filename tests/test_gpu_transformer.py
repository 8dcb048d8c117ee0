"""Transformer block forward on the GPU vs the reference CPU build of the same
graph (oracle/_ref: every op a sil:: array op on Device::CPU), end-to-end
tolerance |g - r| <= 2e-5 (1 + |r|)."""
import numpy as np
import pytest
import torch

from silarray_b200 import gpu, transformer
from oracle import transformer_ref as TR

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
    ref = TR.reference_forward(cfg, p, x)
    TR.check_parity(out.cpu().numpy(), ref, cfg)
    gpu.device_status()


@pytest.mark.parametrize("chunks", [1, 3, 8])
def test_forward_host_chunks(cuda, chunks):
    """forward_host (host buffers, copies overlapped with the compute of other
    sequence groups) gives the device forward's result bit for bit: every
    output element sums the same products in the same order."""
    cfg = transformer.Config(batch=8, seq=256, d_model=256, heads=4, d_ff=1024)
    p = transformer.init_params(cfg, seed=5)
    x = transformer.init_input(cfg, seed=6)
    blk = transformer.Block(cfg, p, device="cuda")
    want = blk.forward(torch.from_numpy(x).cuda()).cpu().numpy()
    xh = torch.from_numpy(x).pin_memory()
    oh = torch.empty(cfg.tokens * cfg.d_model, dtype=torch.float32).pin_memory()
    for _ in range(2):  # the second call reuses the staging buffers and streams
        oh.zero_()
        blk.forward_host(xh, oh, chunks=chunks)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(oh.numpy().reshape(want.shape), want)
    gpu.device_status()


def test_forward_host_stream(cuda):
    """Consecutive batches host to host with the copies of neighbouring
    batches overlapping the compute: each output equals the device forward of
    its input -- bit for bit for the middle batches, and within the block's
    tolerance for the first and the last, which run as two half-batches (their
    GEMMs may take other split-K plans, so other rounding) -- in one call over
    five batches and in five calls of one batch whose outputs alternate
    between two host buffers."""
    from oracle import transformer_ref as TR
    cfg = transformer.Config(batch=4, seq=256, d_model=256, heads=4, d_ff=1024)
    p = transformer.init_params(cfg, seed=7)
    blk = transformer.Block(cfg, p, device="cuda")
    xs = [transformer.init_input(cfg, seed=10 + k) for k in range(5)]
    want = [blk.forward(torch.from_numpy(x).cuda()).cpu().numpy() for x in xs]
    xh = [torch.from_numpy(x).pin_memory() for x in xs]
    oh = [torch.empty(cfg.tokens * cfg.d_model, dtype=torch.float32).pin_memory() for _ in range(5)]

    def same(got, k, exact):
        got = got.reshape(want[k].shape)
        if exact:
            np.testing.assert_array_equal(got, want[k])
        else:
            TR.check_parity(got, want[k].astype(np.float64), cfg)
    blk.forward_host_stream(xh, oh)
    torch.cuda.synchronize()
    for k in range(5):
        same(oh[k].numpy(), k, 0 < k < 4)
    ring = [torch.empty(cfg.tokens * cfg.d_model, dtype=torch.float32).pin_memory() for _ in range(2)]
    got = []
    for k in range(5):  # one batch per call (each both first and last), outputs read back between calls
        blk.forward_host_stream([xh[k]], [ring[k % 2]])
        torch.cuda.synchronize()
        got.append(ring[k % 2].numpy().copy())
    for k in range(5):
        same(got[k], k, False)
    gpu.device_status()


def test_graph_replay_matches_eager(cuda):
    """The second and later forwards over the same buffers replay a CUDA graph
    of the first one's launches: bit for bit the eager result, also after the
    input changes in place, and the replayed kernels are counted."""
    cfg = transformer.Config(batch=2, seq=256, d_model=256, heads=4, d_ff=1024)
    p = transformer.init_params(cfg, seed=8)
    eager = transformer.Block(cfg, p, device="cuda", graphs=False)
    graphed = transformer.Block(cfg, p, device="cuda", graphs=True)
    x = torch.from_numpy(transformer.init_input(cfg, seed=9)).cuda()
    out = torch.empty(cfg.tokens * cfg.d_model, device="cuda")
    for step in range(3):
        if step == 2:
            x.mul_(0.5)  # new content, same buffer: the replay reads it
        want = eager.forward(x).cpu().numpy()
        got = graphed.forward(x, out).cpu().numpy()
        np.testing.assert_array_equal(got, want)
    assert graphed.replayed_launches > 0
    with pytest.raises(ValueError):
        graphed.forward(x.reshape(-1)[: x.numel() // 2], out)
    gpu.device_status()
