"""All-gather through peer memory (CUDA IPC over NVLink) for the split-KV
decode: see srswa_peer_allgather in include/srswa.h.

    ex = PeerAllGather(slot_bytes, group)     # collective set-up, once
    out = ex(payload)                         # [world, *payload.shape] view of this rank's region

Set-up exchanges the regions' IPC handles with one all_gather_object over the
process group (any backend); after that no collective runs.  A call is one
push launch (plain stores into every peer's slot + released flags) and one
bounded wait launch, both capturable in a CUDA graph; ``push`` is the push
alone, for a consumer kernel that waits itself (the library's key merge and
log-sum-exp merge take ``self.peer`` for that), and ``self.peer`` also makes
the router's shard kernel push its keys itself.  A returned view is valid
until the next exchange on the same object overwrites it, so a decode step
alternates two objects (router keys, attention partials).  With ll=True the
object speaks the LL protocol (srswa.h, "peer exchange"): only the fused
kernels (srswa_route_shard_select, srswa_decode_attend_push, srswa_lse_merge)
use it, and ``push`` / ``__call__`` are refused.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L


class PeerAllGather:
    def __init__(self, slot_bytes: int, group=None, device=None, ll: bool = False):
        import torch.distributed as dist
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else device
        self.slot = -(-int(slot_bytes) // 16) * 16
        lib = L.lib()
        size = C.c_size_t(0)
        L.check(lib.srswa_peer_region_size(self.world, self.slot, C.byref(size)), "srswa_peer_region_size")
        self.size = size.value
        reg = C.c_void_p()
        with torch.cuda.device(self.device):
            L.check(lib.srswa_peer_region_alloc(self.size, C.byref(reg)), "srswa_peer_region_alloc")
        self.region = reg.value
        h = (C.c_char * 64)()
        L.check(lib.srswa_peer_ipc_handle(C.c_void_p(self.region), h), "srswa_peer_ipc_handle")
        handles = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(handles, bytes(h), group=group)
        else:
            handles = [bytes(h)]
        self.mapped = []
        ptrs = []
        with torch.cuda.device(self.device):
            for r, hr in enumerate(handles):
                if r == self.rank:
                    ptrs.append(self.region)
                    continue
                p = C.c_void_p()
                L.check(lib.srswa_peer_ipc_open((C.c_char * 64).from_buffer_copy(hr), C.byref(p)),
                        "srswa_peer_ipc_open")
                self.mapped.append(p.value)
                ptrs.append(p.value)
        self.regions = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        self.counter = torch.zeros(1, dtype=torch.int64, device=self.device)
        self.tickets = torch.zeros(2, dtype=torch.int32, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        # the srswa_peer descriptor the library's producers / consumers take
        # ll: the LL protocol (payload words carry the epoch; only the
        # library's fused producers / consumers take it)
        self.ll = bool(ll)
        self.peer = L.Peer(self.regions.data_ptr(), self.region, self.slot, self.rank, self.world,
                           self.counter.data_ptr(), self.tickets.data_ptr(), self.status.data_ptr(),
                           1 if self.ll else 0)
        # this rank's region as bytes: slot r (after the 256-byte flag header) = rank r's payload
        self._slots = _RegionView(self.region, self.size, self.device).tensor[256:].view(self.world, self.slot)

    def _check_payload(self, payload):
        x = payload if payload.is_contiguous() else payload.contiguous()
        nbytes = x.numel() * x.element_size()
        if nbytes > self.slot:
            raise ValueError(f"payload of {nbytes} B exceeds the {self.slot} B slot")
        if nbytes % 16:
            raise ValueError("payload size must be a multiple of 16 bytes")
        return x, nbytes

    def slots(self, shape, dtype) -> torch.Tensor:
        """[world, *shape] view of this rank's region: slot r = rank r's payload."""
        nbytes = torch.Size(shape).numel() * torch.empty(0, dtype=dtype).element_size()
        return self._slots[:, :nbytes].view(dtype).view((self.world,) + tuple(shape))

    def own_slot(self, shape, dtype) -> torch.Tensor:
        """View of this rank's own slot in its own region: a producer kernel
        that pushes itself (srswa_decode_attend_push) writes its payload here."""
        nbytes = torch.Size(shape).numel() * torch.empty(0, dtype=dtype).element_size()
        return self._slots[self.rank, :nbytes].view(dtype).view(tuple(shape))

    def push(self, payload: torch.Tensor) -> torch.Tensor:
        """Producer half only (one launch); a consumer kernel given
        ``self.peer`` as its wait reads the returned view."""
        x, nbytes = self._check_payload(payload)
        L.check(L.lib().srswa_peer_push(x.data_ptr(), nbytes, C.byref(self.peer), L.stream_of(x)), "srswa_peer_push")
        return self.slots(x.shape, x.dtype)

    def __call__(self, payload: torch.Tensor) -> torch.Tensor:
        """Push + wait (two launches): the gathered [world, *payload.shape]."""
        x, nbytes = self._check_payload(payload)
        L.check(L.lib().srswa_peer_allgather(x.data_ptr(), nbytes, C.byref(self.peer), L.stream_of(x)),
                "srswa_peer_allgather")
        return self.slots(x.shape, x.dtype)

    def check(self):
        """Raise if a bounded wait expired (reads the device status: syncs)."""
        if int(self.status.item()):
            raise L.SrswaError(f"peer all-gather: a wait for a peer expired (code {int(self.status.item())})")

    def close_mappings(self):
        """Unmap the peers' regions (after every rank's GPU work is done)."""
        lib = L.lib()
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            for p in self.mapped:
                lib.srswa_peer_ipc_close(C.c_void_p(p))
            self.mapped = []

    def close(self):
        """Unmap the peers and free this rank's region (after every peer has
        unmapped it: call close_mappings on all ranks, a barrier, then close)."""
        self.close_mappings()
        self._slots = None
        if self.region:
            with torch.cuda.device(self.device):
                L.lib().srswa_peer_region_free(C.c_void_p(self.region))
            self.region = None


class _RegionView:
    """A uint8 CUDA tensor over memory this library allocated (no ownership:
    the PeerAllGather object frees it)."""

    def __init__(self, ptr, size, device):
        class _Iface:
            __cuda_array_interface__ = {"shape": (size,), "typestr": "|u1", "data": (ptr, False), "version": 3,
                                        "strides": None}
        with torch.cuda.device(device):
            self.tensor = torch.as_tensor(_Iface(), device=device)
