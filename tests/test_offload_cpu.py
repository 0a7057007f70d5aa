"""Block offload on CPU: the reference's own offload tests (tests/test_block_offload_cpu.py)
run against this offloader, plus arena packing checks."""
from __future__ import annotations

import pytest
import torch
from torch import nn

from krea2_svdquant_b200.offload import TransformerBlockOffloader, _BlockArena, enable_block_offload


class _Block(nn.Module):
    def __init__(self, dim: int):
        super().__init__()
        self.lin = nn.Linear(dim, dim)
        self.register_buffer("scale", torch.ones(dim))

    def forward(self, x):
        return self.lin(x) * self.scale


class _Toy(nn.Module):
    def __init__(self, dim: int, num_blocks: int):
        super().__init__()
        self.embed = nn.Linear(dim, dim)
        self.transformer_blocks = nn.ModuleList([_Block(dim) for _ in range(num_blocks)])
        self.norm_out = nn.Linear(dim, dim)

    def forward(self, x):
        x = self.embed(x)
        for block in self.transformer_blocks:
            x = block(x)
        return self.norm_out(x)


def _make_pair(dim=8, num_blocks=5):
    torch.manual_seed(0)
    ref = _Toy(dim, num_blocks)
    swapped = _Toy(dim, num_blocks)
    swapped.load_state_dict(ref.state_dict())
    return ref, swapped


def test_block_offload_matches_reference_cpu():
    ref, swapped = _make_pair()
    x = torch.randn(2, 8)
    expected = ref(x)
    off = enable_block_offload(swapped, "cpu", num_blocks_on_gpu=2)
    assert off.num_blocks == 5
    assert off.attr_names == ["transformer_blocks"]
    assert torch.allclose(expected, swapped(x), atol=1e-6)


def test_resident_window_bounded_and_cleanup():
    _, swapped = _make_pair(num_blocks=6)
    off = TransformerBlockOffloader(swapped, "cpu", num_blocks_on_gpu=2).install()
    swapped(torch.randn(1, 8))
    assert len(off._resident) <= 2
    off.remove()
    assert len(off._resident) == 0
    assert len(off._handles) == 0
    assert all(p.device.type == "cpu" for p in swapped.transformer_blocks.parameters())


def test_missing_container_raises():
    with pytest.raises(ValueError):
        TransformerBlockOffloader(nn.Linear(4, 4), "cpu")


def test_prefetch_needs_cuda_device():
    _, swapped = _make_pair()
    with pytest.raises(ValueError):
        TransformerBlockOffloader(swapped, "cpu", prefetch=True)


def test_arena_packs_block_into_one_buffer():
    torch.manual_seed(1)
    blk = _Block(24)
    blk.extra = nn.Parameter(torch.randn(3, 5).to(torch.bfloat16))
    blk.register_buffer("codes", torch.randint(0, 255, (7,), dtype=torch.uint8))
    before = {k: v.clone() for k, v in blk.state_dict().items()}
    arena = _BlockArena(blk, pin=False)
    after = blk.state_dict()
    for k, v in before.items():
        assert torch.equal(after[k], v) and after[k].dtype == v.dtype
    # every tensor is a view into the arena, at a 256-byte aligned offset
    base = arena.host.data_ptr()
    for t in after.values():
        off = t.data_ptr() - base
        assert 0 <= off < arena.nbytes and off % 256 == 0
    # a second buffer with the same layout reproduces the block
    other = torch.zeros_like(arena.host)
    other.copy_(arena.host)
    arena.attach_device(other)
    for k, v in before.items():
        assert torch.equal(blk.state_dict()[k], v)
    arena.attach_cpu()
    assert blk.lin.weight.data_ptr() - base >= 0


def test_multiple_containers():
    class Two(nn.Module):
        def __init__(self):
            super().__init__()
            self.transformer_blocks = nn.ModuleList([_Block(4), _Block(4)])
            self.single_transformer_blocks = nn.ModuleList([_Block(4)])

        def forward(self, x):
            for b in list(self.transformer_blocks) + list(self.single_transformer_blocks):
                x = b(x)
            return x

    torch.manual_seed(0)
    m = Two()
    x = torch.randn(3, 4)
    want = m(x)
    off = enable_block_offload(m, "cpu")
    assert off.num_blocks == 3 and off.attr_names == ["transformer_blocks", "single_transformer_blocks"]
    assert torch.allclose(m(x), want)
