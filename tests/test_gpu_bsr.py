"""Batched block-sparse propagation on the tensor cores (tcgen05) against a
plain PyTorch fp32 block product of the same bf16 weights and spikes.
Tolerance: 1e-2 relative to the largest reference current (the batched
microbenchmark's bar); bf16 x {0,1} products are exact in fp32, so only the
summation order differs."""
import pytest
import torch

from libnrn_b200 import bsr as B

pytestmark = pytest.mark.gpu
TOL = 1e-2


def rel(a, b):
    return float((a - b).abs().max()) / max(1e-30, float(b.abs().max()))


def test_small_with_empty_and_long_rows():
    torch.manual_seed(0)
    dev = "cuda"
    nr, nc = 12, 20
    # row 0 empty, row 1 every column (more blocks than pipeline stages), others random
    rows = [[], list(range(nc))] + [sorted(torch.randperm(nc)[:k].tolist()) for k in (3, 1, 7, 0, 5, 2, 9, 4, 6, 8)]
    cols = [c for r in rows for c in r]
    row_ptr = torch.tensor([0] + [len(r) for r in rows]).cumsum(0)
    blocks = (torch.randn(len(cols), 64, 64, device=dev) * 0.02).to(torch.bfloat16)
    w = B.BlockSparse(row_ptr, torch.tensor(cols), blocks, nr, nc)
    s = (torch.rand(nc * 64, 64, device=dev) < 0.05).float()
    tiles = B.spike_tiles(nc)
    B.pack_spikes(s, tiles)
    assert torch.equal(B.unpack_spikes(tiles), s)
    i0 = torch.randn(nr * 64, 64, device=dev)
    i = i0.clone()
    w.propagate(tiles, i)
    torch.cuda.synchronize()
    w.check()
    ref = i0 + B.reference_product(w, blocks, s)
    assert rel(i, ref) <= TOL
    assert torch.equal(i[:64], i0[:64])          # the empty row is untouched


def test_batched_config_scaled_down():
    # the 2%-density, p=0.01 configuration at 32,768 x 32,768 neurons
    w = B.BlockSparse.random(32768, 32768, 0.02, seed=4, keep_blocks=True)
    tiles = B.spike_tiles(w.n_pre_blocks)
    i = torch.zeros(32768, 64, device="cuda")
    ref = torch.zeros_like(i)
    for step in range(3):
        B.bernoulli_spikes(tiles, seed=5, step=step, p=0.01)
        s = B.unpack_spikes(tiles)
        w.propagate(tiles, i)
        ref += B.reference_product(w, w.blocks, s)
    torch.cuda.synchronize()
    w.check()
    assert rel(i, ref) <= TOL


def test_spike_generator():
    tiles = B.spike_tiles(64)
    B.bernoulli_spikes(tiles, seed=5, step=7, p=0.01)
    s1 = B.unpack_spikes(tiles)
    B.bernoulli_spikes(tiles, seed=5, step=7, p=0.01)
    assert torch.equal(B.unpack_spikes(tiles), s1)          # keyed, not stateful
    B.bernoulli_spikes(tiles, seed=5, step=8, p=0.01)
    assert not torch.equal(B.unpack_spikes(tiles), s1)
    assert set(s1.unique().tolist()) <= {0.0, 1.0}
    m = float(s1.mean())
    assert abs(m - 0.01) < 0.002                            # 262,144 draws
