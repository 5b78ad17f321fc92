"""IPC-shared ("symmetric") device buffers: every rank holds one allocation and maps every peer's.

``SymmetricBuffer(nbytes, group)`` allocates ``nbytes`` on this rank's GPU with
``cudaMalloc`` (native extension), exchanges the CUDA IPC handles over the
process group and opens the peers' allocations, so ``ptrs[q]`` is rank q's
buffer as an address valid in THIS process.  Kernels in ``csrc/symm.cu`` read
and write those addresses directly over NVLink.  ``view(offset, shape, dtype)``
is a non-owning tensor over the local allocation; the buffer must outlive its
views.  ``close()`` is collective: every rank unmaps its peers' buffers, then a
barrier, then every rank frees its own allocation.
"""

from __future__ import annotations

from typing import List, Optional, Sequence

import torch
import torch.distributed as dist

from vlmrl.ops._ext import ext


class SymmetricBuffer:
    def __init__(self, nbytes: int, group=None, device: Optional[torch.device] = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.dev_index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.nbytes = int(nbytes)
        self.local = int(ext().symm_alloc(max(self.nbytes, 256), self.dev_index))
        handle = bytes(ext().symm_ipc_handle(self.local, self.dev_index).numpy().tobytes())
        handles: List[Optional[bytes]] = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        self.ptrs: List[int] = []
        for q, h in enumerate(handles):
            if q == self.rank:
                self.ptrs.append(self.local)
            else:
                t = torch.frombuffer(bytearray(h), dtype=torch.uint8)
                self.ptrs.append(int(ext().symm_open(t, self.dev_index)))
        self.closed = False

    def view(self, offset_bytes: int, shape: Sequence[int], dtype: torch.dtype) -> torch.Tensor:
        numel = 1
        for s in shape:
            numel *= int(s)
        end = int(offset_bytes) + numel * torch.empty((), dtype=dtype).element_size()
        if end > self.nbytes:
            raise ValueError(f"view [{offset_bytes}, {end}) exceeds the {self.nbytes}-byte buffer")
        return ext().symm_view(self.local, int(offset_bytes), [int(s) for s in shape], dtype, self.dev_index)

    def close(self) -> None:
        if self.closed:
            return
        torch.cuda.synchronize(self.device)
        for q, p in enumerate(self.ptrs):
            if q != self.rank:
                ext().symm_close(p, self.dev_index)
        dist.barrier(group=self.group)
        ext().symm_free(self.local, self.dev_index)
        self.closed = True


def p2p_supported(group=None) -> bool:
    """NCCL process group with every rank on one node and peer access between this GPU and all others."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_backend(group) != "nccl":
        return False
    if not torch.cuda.is_available():
        return False
    dev = torch.cuda.current_device()
    ok = torch.tensor([1], device="cuda")
    local = torch.cuda.device_count()
    world = dist.get_world_size(group)
    if world > local:
        ok.zero_()
    else:
        for q in range(local):
            if q != dev and not torch.cuda.can_device_access_peer(dev, q):
                ok.zero_()
    dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
    return bool(ok.item())


__all__ = ["SymmetricBuffer", "p2p_supported"]
