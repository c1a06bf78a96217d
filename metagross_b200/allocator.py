"""Page allocators.

``BlockAllocator`` is the host allocator of the reference's per-sequence cache
(metagross/allocator.py:1-33), same interface and errors: a LIFO free list
initialised to ``range(num_pages)``; ``allocate()`` pops the LAST id (a fresh
allocator hands out N-1, N-2, ...), ``free()`` appends, exhaustion and double
free raise RuntimeError, an id outside ``[0, num_pages)`` raises ValueError.
Membership is tracked in a set, so ``free`` is O(1) instead of the
reference's O(N) list scan; the observable order is identical.

``DeviceBlockAllocator`` holds the same LIFO stack in device memory for the
batched cache; the kernels that pop and push it (``_C.plan_append``,
``_C.free_sequences``) preserve the reference's order: ids are handed out in
(sequence index, logical page) order and freed in (listed sequence,
block-table) order.
"""
from __future__ import annotations

import torch


class BlockAllocator:
    def __init__(self, num_pages):
        if num_pages <= 0:
            raise ValueError("num_pages must be positive")
        self.num_pages = num_pages
        self._free = list(range(num_pages))
        self._free_set = set(self._free)

    def allocate(self) -> int:
        if not self._free:
            raise RuntimeError(
                f"BlockAllocator out of pages (all {self.num_pages} in use). "
                "Increase max_pages or free finished sequences."
            )
        p = self._free.pop()
        self._free_set.discard(p)
        return p

    def free(self, page_idx) -> None:
        if not (0 <= page_idx < self.num_pages):
            raise ValueError(f"page_idx {page_idx} out of range [0, {self.num_pages})")
        if page_idx in self._free_set:
            raise RuntimeError(f"page_idx {page_idx} is already free (double free)")
        self._free.append(page_idx)
        self._free_set.add(page_idx)

    @property
    def num_free(self) -> int:
        return len(self._free)

    @property
    def num_used(self) -> int:
        return self.num_pages - len(self._free)


class DeviceBlockAllocator:
    """LIFO page stack in device memory (int32 free_stack [N], n_free [1], in_use [N])."""

    def __init__(self, num_pages: int, device="cuda"):
        if num_pages <= 0:
            raise ValueError("num_pages must be positive")
        self.num_pages = int(num_pages)
        self.device = torch.device(device)
        self.free_stack = torch.empty(self.num_pages, dtype=torch.int32, device=self.device)
        self.n_free = torch.empty(1, dtype=torch.int32, device=self.device)
        self.in_use = torch.empty(self.num_pages, dtype=torch.int32, device=self.device)
        self.reset()

    def reset(self) -> None:
        from . import _C

        _C.alloc_init(self.free_stack, self.n_free, self.in_use)

    @property
    def num_free(self) -> int:
        """Free pages (synchronises with the device)."""
        return int(self.n_free.item())

    @property
    def num_used(self) -> int:
        return self.num_pages - self.num_free

    def free_list(self) -> list[int]:
        """The stack, bottom to top (synchronises); the next allocation is the last element."""
        n = self.num_free
        return self.free_stack[:n].tolist()
