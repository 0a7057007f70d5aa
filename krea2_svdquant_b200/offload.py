"""Transformer-block offload with a native prefetcher
(API of src/krea2_svdquant/runtime/block_offload.py:75-213).

The non-block modules live on the device; transformer blocks live in host
memory and come to the device only around their forward, with at most
``num_blocks_on_gpu`` blocks resident after a pass (the reference's contract,
block_offload.py:157-173).

On a CUDA device the blocks move differently from the reference, which calls
``.to(device)`` per tensor on the compute stream:

* each block's parameters and buffers are packed once into one pinned host
  arena, which becomes the block's CPU master copy;
* ``num_blocks_on_gpu + 1`` device slots hold resident blocks; a block's upload
  is one ``cudaMemcpyAsync`` of its arena into a slot on the prefetcher's
  low-priority copy stream (``svdq_prefetch_*`` in the C ABI);
* while block *i* runs, block *i + 1* (in container order, wrapping to the
  first block for the next denoising step) is uploaded, and its
  ``SVDQuantLinear`` layers derive their fp16 GEMM operands on the copy stream
  too, so the next block starts with everything ready;
* the compute stream waits for an upload on the GPU (an event), not on the
  host; a slot is reused only after the compute stream has released it.

On a CPU device the offloader keeps the reference's plain swap semantics.
"""
from __future__ import annotations

import ctypes
from collections import deque
from collections.abc import Iterable, Sequence

import torch
from torch import nn

DEFAULT_BLOCK_ATTRS: tuple[str, ...] = ("transformer_blocks", "single_transformer_blocks")
_ALIGN = 256


def _first_cuda_device(args: tuple, kwargs: dict) -> torch.device | None:
    for v in list(args) + list(kwargs.values()):
        if isinstance(v, torch.Tensor) and v.is_cuda:
            return v.device
    return None


class _BlockArena:
    """A block's parameters and buffers packed into one (optionally pinned) host buffer.

    After construction the block's CPU tensors are views into ``host``, so the
    packed copy is the only host copy.  ``attach_device(base)`` points the block
    at the same layout over a device buffer, ``attach_cpu()`` back at ``host``."""

    def __init__(self, block: nn.Module, *, pin: bool):
        self.block = block
        block.to("cpu")
        params: list[tuple[nn.Parameter, torch.Tensor]] = []
        seen: set[int] = set()
        for p in block.parameters(recurse=True):
            if id(p) not in seen:
                seen.add(id(p))
                params.append((p, p.data))
        bufs: list[tuple[nn.Module, str, torch.Tensor]] = []
        for m in block.modules():
            for name, b in m._buffers.items():
                if b is not None:
                    bufs.append((m, name, b))
        self._layout: list[tuple[int, int, torch.dtype, torch.Size]] = []
        off = 0
        for t in [t for _, t in params] + [t for _, _, t in bufs]:
            nbytes = t.numel() * t.element_size()
            self._layout.append((off, nbytes, t.dtype, t.shape))
            off += (nbytes + _ALIGN - 1) // _ALIGN * _ALIGN
        self.nbytes = off
        self.host = torch.empty(max(off, 1), dtype=torch.uint8, pin_memory=pin)
        views = self._views(self.host)
        src = [t for _, t in params] + [t for _, _, t in bufs]
        for v, t in zip(views, src):
            v.copy_(t.contiguous())
        self._params = params
        self._bufs = bufs
        self._cpu_views = views
        self._attach(views)

    def _views(self, base: torch.Tensor) -> list[torch.Tensor]:
        out = []
        for off, nbytes, dtype, shape in self._layout:
            out.append(base[off:off + nbytes].view(dtype).view(shape))
        return out

    def _attach(self, views: list[torch.Tensor]) -> None:
        n = len(self._params)
        for (p, _), v in zip(self._params, views[:n]):
            p.data = v
        for (m, name, _), v in zip(self._bufs, views[n:]):
            m._buffers[name] = v

    def attach_device(self, base: torch.Tensor) -> None:
        self._attach(self._views(base))

    def attach_cpu(self) -> None:
        self._attach(self._cpu_views)

    def to_device_plain(self, device: torch.device, non_blocking: bool) -> None:
        self._attach([v.to(device, non_blocking=non_blocking) for v in self._cpu_views])


def _svdq_layers(block: nn.Module):
    from .linear import SVDQuantLinear
    return [m for m in block.modules() if isinstance(m, SVDQuantLinear)]


class TransformerBlockOffloader:
    """Keep transformer blocks in host memory and stream them to the device per forward."""

    def __init__(self, transformer: nn.Module, device: torch.device | str, *, num_blocks_on_gpu: int = 1,
                 pin_memory: bool = False, block_attrs: Sequence[str] | None = None,
                 prefetch: bool | None = None, wait_timeout_ms: int = -1):
        self.transformer = transformer
        self.device = torch.device(device)
        self.num_blocks_on_gpu = max(1, int(num_blocks_on_gpu))
        self.pin_memory = bool(pin_memory)
        self.prefetch = (self.device.type == "cuda") if prefetch is None else bool(prefetch)
        if self.prefetch and self.device.type != "cuda":
            raise ValueError("prefetching offload needs a CUDA device")
        self.wait_timeout_ms = int(wait_timeout_ms)
        self._handles: list = []
        self._arenas: dict[int, _BlockArena] = {}
        self._order: list[int] = []
        self._resident: deque[int] = deque()
        self._containers = self._find_containers(block_attrs)
        if not self._containers:
            raise ValueError(f"no transformer block containers found; expected one of "
                             f"{block_attrs or DEFAULT_BLOCK_ATTRS}")
        # prefetch state
        self._pf = None
        self._copy_stream: torch.cuda.ExternalStream | None = None
        self._slots: list[torch.Tensor] = []
        self._slot_of: dict[int, int] = {}     # block key -> slot
        self._slot_owner: dict[int, int] = {}  # slot -> block key
        self._slot_lru: deque[int] = deque()

    # ---------------------------------------------------------------- reference API
    @property
    def num_blocks(self) -> int:
        return sum(len(b) for _, b in self._containers)

    @property
    def attr_names(self) -> list[str]:
        return [a for a, _ in self._containers]

    def _find_containers(self, block_attrs: Sequence[str] | None) -> list[tuple[str, nn.ModuleList]]:
        found = []
        for attr in tuple(block_attrs) if block_attrs else DEFAULT_BLOCK_ATTRS:
            c = getattr(self.transformer, attr, None)
            if isinstance(c, nn.ModuleList) and len(c) > 0:
                found.append((attr, c))
        return found

    def _iter_blocks(self) -> Iterable[nn.Module]:
        for _, c in self._containers:
            yield from c

    def _move_non_blocks_to_device(self) -> None:
        saved = list(self._containers)
        for attr, _ in saved:
            setattr(self.transformer, attr, None)
        try:
            self.transformer.to(self.device)
        finally:
            for attr, c in saved:
                setattr(self.transformer, attr, c)

    def install(self) -> "TransformerBlockOffloader":
        self._move_non_blocks_to_device()
        pin = (self.pin_memory or self.prefetch) and torch.cuda.is_available()
        for block in self._iter_blocks():
            self._arenas[id(block)] = _BlockArena(block, pin=pin)
            self._order.append(id(block))
            self._handles.append(block.register_forward_pre_hook(self._pre_hook, with_kwargs=True))
            self._handles.append(block.register_forward_hook(self._post_hook))
        if self.prefetch:
            self._start_prefetcher()
        if torch.cuda.is_available():
            torch.cuda.empty_cache()
        return self

    def offload_all(self) -> None:
        """Return every block to host memory and drop the resident window."""
        if self._pf is not None:
            from . import _lib
            _lib.check(_lib.lib().svdq_prefetcher_sync(self._pf, -1))
        for key, arena in self._arenas.items():
            self._evict(key)
        self._resident.clear()
        if torch.cuda.is_available():
            torch.cuda.empty_cache()

    def remove(self) -> None:
        """Remove the hooks, return blocks to host memory and free the device slots."""
        for h in self._handles:
            h.remove()
        self._handles.clear()
        self.offload_all()
        self._stop_prefetcher()

    # ---------------------------------------------------------------- swapping
    def _evict(self, key: int) -> None:
        arena = self._arenas[key]
        for m in _svdq_layers(arena.block):
            m.release_prepared()
        arena.attach_cpu()
        slot = self._slot_of.pop(key, None)
        if slot is not None:
            self._slot_owner.pop(slot, None)

    def _pre_hook(self, block: nn.Module, args: tuple, kwargs: dict):
        key = id(block)
        if self.prefetch:
            self._make_resident_prefetch(key)
            self._prefetch_next(key)
        else:
            device = _first_cuda_device(args, kwargs) or self.device
            if key not in self._resident:
                self._arenas[key].to_device_plain(device, non_blocking=self.pin_memory)
        if key in self._resident:
            self._resident.remove(key)
        self._resident.append(key)
        while len(self._resident) > self.num_blocks_on_gpu:
            old = self._resident.popleft()
            if old == key:
                self._resident.append(old)
                break
            if not self.prefetch:
                self._evict(old)
        return None

    def _post_hook(self, block: nn.Module, args, output):
        if self.prefetch:
            slot = self._slot_of.get(id(block))
            if slot is not None:
                from . import _lib
                stream = torch.cuda.current_stream(self.device).cuda_stream
                _lib.check(_lib.lib().svdq_prefetch_release(self._pf, slot, ctypes.c_void_p(stream)))
        return None

    # ---------------------------------------------------------------- prefetch path
    def _start_prefetcher(self) -> None:
        from . import _lib
        n_slots = self.num_blocks_on_gpu + 1
        h = ctypes.c_void_p()
        index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.device = torch.device("cuda", index)
        _lib.check(_lib.lib().svdq_prefetcher_create(index, n_slots, ctypes.byref(h)))
        self._pf = h
        s = ctypes.c_void_p()
        _lib.check(_lib.lib().svdq_prefetcher_copy_stream(self._pf, ctypes.byref(s)))
        self._copy_stream = torch.cuda.ExternalStream(s.value, device=self.device)
        slot_bytes = max(a.nbytes for a in self._arenas.values())
        self._slots = [torch.empty(slot_bytes, dtype=torch.uint8, device=self.device) for _ in range(n_slots)]
        self._slot_lru = deque(range(n_slots))

    def _stop_prefetcher(self) -> None:
        if self._pf is not None:
            from . import _lib
            _lib.check(_lib.lib().svdq_prefetcher_destroy(self._pf))
            self._pf = None
        self._slots = []
        self._slot_of.clear()
        self._slot_owner.clear()
        self._copy_stream = None

    def _claim_slot(self, key: int, protect: set[int]) -> int:
        """A slot for block ``key``: a free one, else the least recently used one whose
        block is not in ``protect`` (that block is evicted)."""
        for slot in list(self._slot_lru):
            owner = self._slot_owner.get(slot)
            if owner is None or owner not in protect:
                if owner is not None:
                    self._evict(owner)
                    if owner in self._resident:
                        self._resident.remove(owner)
                self._slot_lru.remove(slot)
                self._slot_lru.append(slot)
                return slot
        raise RuntimeError("block offload: no device slot can be reused")

    def _upload(self, key: int, slot: int) -> None:
        from . import _lib
        arena = self._arenas[key]
        base = self._slots[slot]
        L = _lib.lib()
        _lib.check(L.svdq_prefetch_begin(self._pf, slot, ctypes.c_void_p(base.data_ptr()),
                                         ctypes.c_void_p(arena.host.data_ptr()), arena.nbytes))
        arena.attach_device(base)
        self._slot_of[key] = slot
        self._slot_owner[slot] = key
        layers = _svdq_layers(arena.block)
        if layers:
            compute = torch.cuda.current_stream(self.device)
            with torch.cuda.stream(self._copy_stream):
                for m in layers:
                    prep = m.prepare(self.device)
                    for t in vars(prep).values():
                        if isinstance(t, torch.Tensor) and t.is_cuda:
                            t.record_stream(compute)
        _lib.check(L.svdq_prefetch_commit(self._pf, slot))

    def _make_resident_prefetch(self, key: int) -> None:
        from . import _lib
        slot = self._slot_of.get(key)
        if slot is None:
            slot = self._claim_slot(key, protect={key})
            self._upload(key, slot)
        else:
            self._slot_lru.remove(slot)
            self._slot_lru.append(slot)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(_lib.lib().svdq_prefetch_wait(self._pf, slot, ctypes.c_void_p(stream), self.wait_timeout_ms))

    def _prefetch_next(self, key: int) -> None:
        i = self._order.index(key)
        nxt = self._order[(i + 1) % len(self._order)]
        if nxt == key or nxt in self._slot_of:
            return
        # never evict the running block or the blocks inside the resident window
        protect = {key} | set(list(self._resident)[-(self.num_blocks_on_gpu - 1):] if self.num_blocks_on_gpu > 1
                              else [])
        slot = self._claim_slot(nxt, protect=protect)
        self._upload(nxt, slot)


def enable_block_offload(transformer: nn.Module, device: torch.device | str, *, num_blocks_on_gpu: int = 1,
                         pin_memory: bool = False, block_attrs: Sequence[str] | None = None,
                         prefetch: bool | None = None) -> TransformerBlockOffloader:
    """Install transformer-block offload and return the live offloader (block_offload.py:191-213)."""
    return TransformerBlockOffloader(transformer, device, num_blocks_on_gpu=num_blocks_on_gpu,
                                     pin_memory=pin_memory, block_attrs=block_attrs, prefetch=prefetch).install()
