"""Peer mailboxes for sequence parallelism: one device buffer per rank, mapped into every
rank of the node through CUDA IPC, written by peers with direct NVLink stores
(libhdcmamba_b200 ``hdc_peer_*``).

A rank stores its data into a peer's mailbox and raises a generation flag there; the peer
waits (bounded) for the flag before the kernels that read the data.  Every rank bumps its
generation counter once per forward and ends the forward with a flag barrier, so no rank
overwrites a region of the next forward while a slower rank still reads it.
"""
import ctypes

import torch
import torch.distributed as dist

from . import _lib


class _DeviceBytes:
    """__cuda_array_interface__ over raw device memory, for a zero-copy torch view."""

    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3}


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


class PeerMailbox:
    """``nbytes`` of device memory on this rank, mapped into every rank of ``group``.

    ``buf`` is a uint8 tensor over the local mailbox; ``bases`` holds every rank's mailbox
    address as mapped in this process (a device int64 tensor); ``gen`` is the generation
    counter.  Construction is collective (the IPC handles are all-gathered)."""

    def __init__(self, nbytes, group=None, device=None):
        self.lib = _lib.load()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.nbytes = (int(nbytes) + 255) // 256 * 256
        # one rank per GPU: a rank's flag wait spins until another GPU's kernel stores the
        # flag, which two ranks sharing one GPU could not guarantee
        uuids = [None] * self.world
        dist.all_gather_object(uuids, str(torch.cuda.get_device_properties(self.device).uuid), group=group)
        if len(set(uuids)) != self.world:
            raise RuntimeError("peer mailboxes need one rank per GPU; ranks share a device: " + ", ".join(uuids))
        with torch.cuda.device(self.device):
            ptr = ctypes.c_void_p()
            _lib.call("hdc_peer_alloc", self.nbytes, ctypes.byref(ptr))
            self._ptr = ptr
            hb = self.lib.hdc_ipc_handle_bytes()
            raw = (ctypes.c_char * hb)()
            _lib.call("hdc_ipc_handle", ptr, raw)
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(raw), group=group)
            self._opened = []
            bases = []
            for s, hnd in enumerate(handles):
                if s == self.rank:
                    bases.append(ptr.value)
                    continue
                p = ctypes.c_void_p()
                _lib.call("hdc_ipc_open", ctypes.create_string_buffer(hnd, hb), ctypes.byref(p))
                self._opened.append(p)
                bases.append(p.value)
            self.bases = torch.tensor(bases, dtype=torch.int64, device=self.device)
            self.gen = torch.zeros(1, dtype=torch.int32, device=self.device)
            # per-target slice counters of hdc_peer_put, one array per put site that may run
            # concurrently with another (``lane``)
            self.counters = torch.zeros(4, self.world, dtype=torch.int32, device=self.device)
            self.buf = torch.as_tensor(_DeviceBytes(ptr.value, self.nbytes), device=self.device)

    def view(self, offset, shape, dtype):
        """A tensor over the local mailbox at byte ``offset``."""
        n = 1
        for d in shape:
            n *= d
        nb = n * torch.empty((), dtype=dtype).element_size()
        return self.buf[offset:offset + nb].view(dtype).view(*shape)

    def put(self, src, dst_off, flag_off, targets, lane=0):
        """Copy the contiguous tensor ``src`` to byte ``dst_off`` of the mailboxes of the
        ranks in ``targets`` and raise their flag at byte ``flag_off``.  Puts that can run at
        the same time (on different streams) pass different ``lane`` s (0..3)."""
        mask = 0
        for t in targets:
            mask |= 1 << t
        if mask == 0:
            return
        _lib.call("hdc_peer_put", ctypes.c_void_p(src.data_ptr()), src.numel() * src.element_size(),
                  ctypes.c_void_p(self.bases.data_ptr()), dst_off, flag_off, mask, self.world,
                  ctypes.c_void_p(self.gen.data_ptr()), ctypes.c_void_p(self.counters[lane].data_ptr()),
                  _stream(self.device))

    def wait(self, flag_off, sources):
        """Wait until the uint32 flags at byte ``flag_off`` + 4*s (s in ``sources``) of the
        local mailbox reach this rank's generation."""
        mask = 0
        for s in sources:
            mask |= 1 << s
        if mask == 0:
            return
        _lib.call("hdc_peer_wait", ctypes.c_void_p(self._ptr.value + flag_off), mask,
                  ctypes.c_void_p(self.gen.data_ptr()), _stream(self.device))

    def flag_address(self, flag_off):
        """(address of the local uint32 flag at byte ``flag_off``, address of the generation
        counter): for kernels that wait for the flag themselves."""
        return self._ptr.value + flag_off, self.gen.data_ptr()

    def next_generation(self):
        _lib.call("hdc_peer_gen_bump", ctypes.c_void_p(self.gen.data_ptr()), _stream(self.device))

    def barrier(self, bar_off):
        _lib.call("hdc_peer_barrier", ctypes.c_void_p(self.bases.data_ptr()), bar_off, self.world, self.rank,
                  ctypes.c_void_p(self._ptr.value + bar_off), ctypes.c_void_p(self.gen.data_ptr()),
                  _stream(self.device))

    def close(self):
        """Unmap the peers' mailboxes, wait for every rank to do the same, free ours."""
        if self._ptr is None:
            return
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            _lib.call("hdc_ipc_close", p)
        self._opened = []
        dist.barrier(group=self.group)
        self.buf = None
        _lib.call("hdc_peer_free", self._ptr)
        self._ptr = None
