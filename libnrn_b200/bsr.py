"""Batched block-sparse synaptic propagation (64 trials) through the C ABI's
nrn_cuda_bsr_* entry points: 64x64 bf16 weight blocks in block-row CSR,
spikes of 64 independent trials, fp32 input currents [post][trial]."""
from __future__ import annotations

import ctypes as C

import torch

from . import _native as N

BLOCK = 64
TRIALS = 64


def _stream(stream=None) -> C.c_void_p:
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


class BlockSparse:
    """Weights W of n_post x n_pre neurons as 64x64 bf16 blocks; the device
    arrays are owned by this object."""

    def __init__(self, row_ptr: torch.Tensor, col_idx: torch.Tensor, blocks: torch.Tensor,
                 n_post_blocks: int, n_pre_blocks: int):
        dev = blocks.device
        self.n_post_blocks, self.n_pre_blocks = int(n_post_blocks), int(n_pre_blocks)
        self.row_ptr = row_ptr.to(dev, torch.int32).contiguous()
        self.col_idx = col_idx.to(dev, torch.int32).contiguous()
        self.n_blocks = int(self.col_idx.numel())
        blocks = blocks.to(torch.bfloat16).contiguous()
        self.tiles = torch.empty_like(blocks)
        if self.n_blocks:
            N.check(N.lib().nrn_cuda_bsr_pack(C.c_void_p(blocks.data_ptr()), self.n_blocks,
                                              C.c_void_p(self.tiles.data_ptr()), _stream()), "nrn_cuda_bsr_pack")
        self.desc = N.Bsr()
        self.desc.n_post_blocks, self.desc.n_pre_blocks = self.n_post_blocks, self.n_pre_blocks
        self.desc.n_blocks = self.n_blocks
        self.desc.row_ptr = self.row_ptr.data_ptr()
        self.desc.col_idx = self.col_idx.data_ptr()
        self.desc.tiles = self.tiles.data_ptr()
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)

    @classmethod
    def random(cls, n_post: int, n_pre: int, density: float, *, seed: int = 4, std: float = 0.02,
               device="cuda", keep_blocks: bool = False) -> "BlockSparse":
        """Block positions uniform without replacement over the block grid
        (CPU generator seeded with `seed`), values N(0, std) drawn on the
        device (generator seeded with seed + 1), rounded to bf16."""
        nr, nc = n_post // BLOCK, n_pre // BLOCK
        k = int(round(density * nr * nc))
        g = torch.Generator().manual_seed(seed)
        pos = torch.randperm(nr * nc, generator=g)[:k].sort().values
        rows, cols = pos // nc, pos % nc
        row_ptr = torch.zeros(nr + 1, dtype=torch.int64)
        row_ptr[1:] = torch.bincount(rows, minlength=nr).cumsum(0)
        gd = torch.Generator(device=device).manual_seed(seed + 1)
        blocks = (torch.randn(k, BLOCK, BLOCK, generator=gd, device=device) * std).to(torch.bfloat16)
        w = cls(row_ptr, cols, blocks, nr, nc)
        if keep_blocks:
            w.blocks = blocks
        return w

    def propagate(self, spike_tiles: torch.Tensor, i_syn: torch.Tensor, stream=None) -> None:
        """i_syn [n_post][64] += W . S (both on the device)."""
        assert i_syn.dtype == torch.float32 and i_syn.is_contiguous()
        assert i_syn.numel() == self.n_post_blocks * BLOCK * TRIALS
        assert spike_tiles.numel() == self.n_pre_blocks * BLOCK * TRIALS
        N.check(N.lib().nrn_cuda_bsr_propagate(C.byref(self.desc), C.c_void_p(spike_tiles.data_ptr()),
                                               C.c_void_p(i_syn.data_ptr()), C.c_void_p(self.err.data_ptr()),
                                               _stream(stream)), "nrn_cuda_bsr_propagate")

    def check(self) -> None:
        """Raises if a device-side wait of the last propagations timed out."""
        if int(self.err.item()) != 0:
            raise N.NrnError(7, f"nrn_cuda_bsr_propagate: device wait timed out (code {int(self.err.item())})")


def spike_tiles(n_pre_blocks: int, device="cuda") -> torch.Tensor:
    return torch.zeros(n_pre_blocks * BLOCK * TRIALS, dtype=torch.bfloat16, device=device)


def bernoulli_spikes(tiles: torch.Tensor, seed: int, step: int, p: float, stream=None) -> None:
    nb = tiles.numel() // (BLOCK * TRIALS)
    N.check(N.lib().nrn_cuda_bsr_spikes(seed, step, float(p), nb, C.c_void_p(tiles.data_ptr()), _stream(stream)),
            "nrn_cuda_bsr_spikes")


def pack_spikes(s: torch.Tensor, tiles: torch.Tensor) -> None:
    """s: [n_pre][64] 0/1 float32 -> tiles."""
    nb = tiles.numel() // (BLOCK * TRIALS)
    s = s.to(torch.float32).contiguous()
    N.check(N.lib().nrn_cuda_bsr_pack_spikes(C.c_void_p(s.data_ptr()), nb, C.c_void_p(tiles.data_ptr()),
                                             _stream()), "nrn_cuda_bsr_pack_spikes")


def unpack_spikes(tiles: torch.Tensor) -> torch.Tensor:
    nb = tiles.numel() // (BLOCK * TRIALS)
    out = torch.empty(nb * BLOCK, TRIALS, dtype=torch.float32, device=tiles.device)
    N.check(N.lib().nrn_cuda_bsr_unpack_spikes(C.c_void_p(tiles.data_ptr()), nb, C.c_void_p(out.data_ptr()),
                                               _stream()), "nrn_cuda_bsr_unpack_spikes")
    return out


def reference_product(w: BlockSparse, blocks: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """fp32 torch reference: sum over blocks of W_blk.float() @ S[c-block] -> [n_post][64]."""
    rows = torch.repeat_interleave(torch.arange(w.n_post_blocks, device=s.device),
                                   (w.row_ptr[1:] - w.row_ptr[:-1]).long())
    sb = s.view(w.n_pre_blocks, BLOCK, TRIALS)[w.col_idx.long()]
    prod = torch.bmm(blocks.float(), sb)
    out = torch.zeros(w.n_post_blocks, BLOCK, TRIALS, dtype=torch.float32, device=s.device)
    out.index_add_(0, rows, prod)
    return out.view(-1, TRIALS)
