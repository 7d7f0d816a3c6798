"""All-reduce fused with the residual add + RMSNorm of the tensor-parallel
decoder, over CUDA IPC peer memory (``seb_allreduce_add_rmsnorm``).

Each rank owns one peer-memory region holding its ``partial`` (the row-parallel
GEMM's output, written there directly), its ``x`` (the residual stream) and its
``out`` (the normalised rows the next GEMM reads), all ``[n_tokens, hidden]``,
plus the flag words that order the calls. The regions are exchanged once with
CUDA IPC handles over the process group; after that a call is one kernel launch
per rank, with no NCCL and no host synchronisation, and it can be captured in a
CUDA graph.

``PeerAllReduceNorm.single_device(world, ...)`` lays out every rank's region on
one device and runs all ranks' parts in one cooperative launch: the same kernel
and protocol, for testing on one GPU.
"""
from __future__ import annotations

import ctypes

import torch

from . import ops
from ._lib import SEB_MAX_PEERS, SEB_PEER_FLAG_BYTES, SEB_PEER_HANDLE_BYTES, check, lib

_ALIGN = 256


def _round_up(n: int, a: int = _ALIGN) -> int:
    return (n + a - 1) // a * a


class _CudaArray:
    """Exposes a raw device pointer to torch.as_tensor (int16 elements)."""

    def __init__(self, ptr: int, shape):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<i2", "data": (ptr, False),
                                         "version": 2}


def _tensor_at(ptr: int, shape, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    return torch.as_tensor(_CudaArray(ptr, shape), device=device).view(dtype)


def _ptr_array(ptrs) -> ctypes.Array:
    return (ctypes.c_void_p * len(ptrs))(*ptrs)


class PeerAllReduceNorm:
    """x <- x + all_reduce(partial); out <- rmsnorm(x) * weight, on every rank.

    Construct it collectively on every rank of ``group`` (one process per GPU);
    call it in the same order on every rank; ``close()`` it collectively before
    the process group goes away.
    """

    def __init__(self, n_tokens: int, hidden: int, dtype: torch.dtype, device, group=None):
        import torch.distributed as dist

        self._setup(n_tokens, hidden, dtype, device)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 1 <= self.world <= SEB_MAX_PEERS:
            raise ValueError(f"PeerAllReduceNorm: world {self.world} outside [1, {SEB_MAX_PEERS}]")
        self.all_ranks = False
        own = self._alloc()
        handle = (ctypes.c_uint8 * SEB_PEER_HANDLE_BYTES)()
        check("seb_peer_export", lib().seb_peer_export(own, handle))
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=self.device)
        every = torch.empty(self.world * SEB_PEER_HANDLE_BYTES, dtype=torch.uint8, device=self.device)
        dist.all_gather_into_tensor(every, mine, group=group)
        every = bytes(every.cpu().tolist())
        self._imported = []
        bases = []
        # CUDA IPC maps a peer's region into the CURRENT device's context: make
        # it this rank's device whatever the caller's current device is.
        with torch.cuda.device(self.device):
            for q in range(self.world):
                if q == self.rank:
                    bases.append(own)
                    continue
                h = (ctypes.c_uint8 * SEB_PEER_HANDLE_BYTES).from_buffer_copy(
                    every[q * SEB_PEER_HANDLE_BYTES:(q + 1) * SEB_PEER_HANDLE_BYTES])
                p = ctypes.c_void_p()
                check("seb_peer_import", lib().seb_peer_import(h, ctypes.byref(p)))
                self._imported.append(p.value)
                bases.append(p.value)
        self._owned = [own]
        self._bind(bases, local_ranks=[self.rank])
        dist.barrier(group=group)

    @classmethod
    def single_device(cls, world: int, n_tokens: int, hidden: int, dtype: torch.dtype, device):
        """Every rank's region on one device; a call runs all ranks' parts in one
        cooperative launch. ``views(q)`` returns rank q's tensors."""
        self = cls.__new__(cls)
        self._setup(n_tokens, hidden, dtype, device)
        if not 1 <= world <= SEB_MAX_PEERS:
            raise ValueError(f"PeerAllReduceNorm: world {world} outside [1, {SEB_MAX_PEERS}]")
        self.group, self.world, self.rank, self.all_ranks = None, world, 0, True
        self._imported = []
        self._owned = [self._alloc() for _ in range(world)]
        self._bind(self._owned, local_ranks=list(range(world)))
        return self

    # ------------------------------------------------------------------ setup
    def _setup(self, n_tokens, hidden, dtype, device):
        if dtype not in (torch.bfloat16, torch.float16):
            raise ValueError(f"PeerAllReduceNorm: bf16 or fp16 required, got {dtype}")
        if hidden % 8 or hidden > 32768 or n_tokens < 0:
            raise ValueError(f"PeerAllReduceNorm: hidden {hidden} must be a multiple of 8 up to 32768")
        self.n_tokens, self.hidden, self.dtype = int(n_tokens), int(hidden), dtype
        self.device = torch.device(device)
        self.plane = _round_up(max(1, n_tokens * hidden * 2))
        self.region = 3 * self.plane + SEB_PEER_FLAG_BYTES
        self._closed = False

    def _alloc(self) -> int:
        p = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            check("seb_peer_alloc", lib().seb_peer_alloc(self.region, ctypes.byref(p)))
        return p.value

    def _bind(self, bases, local_ranks):
        self._partial = _ptr_array([b for b in bases])
        self._x = _ptr_array([b + self.plane for b in bases])
        self._out = _ptr_array([b + 2 * self.plane for b in bases])
        self._flags = _ptr_array([b + 3 * self.plane for b in bases])
        shape = (self.n_tokens, self.hidden)
        self._views = {q: tuple(_tensor_at(bases[q] + i * self.plane, shape, self.dtype, self.device)
                                for i in range(3)) for q in local_ranks}
        self.partial, self.x, self.out = self._views[local_ranks[0]]

    def views(self, rank: int):
        """(partial, x, out) of `rank` (a rank held on this device)."""
        return self._views[rank]

    # ------------------------------------------------------------------- call
    @ops._nvtx
    def __call__(self, weight: torch.Tensor, eps: float, polls: int = 0) -> torch.Tensor:
        """Sum the ranks' ``partial``, add it to ``x``, RMSNorm into ``out``
        (on every rank); returns ``out``."""
        self._launch(weight, eps, self.rank, self.all_ranks, polls)
        return self.out

    def _launch(self, weight, eps, rank, all_ranks, polls):
        if self._closed:
            raise RuntimeError("PeerAllReduceNorm: closed")
        if weight.device != self.device or weight.dtype != self.dtype or weight.numel() != self.hidden \
                or not weight.is_contiguous():
            raise ValueError(f"PeerAllReduceNorm: weight must be a contiguous [{self.hidden}] {self.dtype} tensor "
                             f"on {self.device}")
        st = lib().seb_allreduce_add_rmsnorm(self._partial, self._x, self._out, self._flags, weight.data_ptr(),
                                             self.n_tokens, self.hidden, float(eps), ops.dtype_code(weight),
                                             int(rank), self.world, int(all_ranks), int(polls),
                                             ops.err_word(self.device).data_ptr(), ops._stream(self.device))
        check("seb_allreduce_add_rmsnorm", st)
        ops.LAUNCHES[0] += 1

    # --------------------------------------------------------------- teardown
    def close(self) -> None:
        """Release the peer memory (collective: every rank calls it)."""
        if self._closed:
            return
        torch.cuda.synchronize(self.device)
        self._views = {}
        self.partial = self.x = self.out = None
        if self.group is not None or not self.all_ranks:
            import torch.distributed as dist

            dist.barrier(group=self.group)  # no peer reads or writes this rank's region any more
            with torch.cuda.device(self.device):  # the mappings live in this device's context
                for p in self._imported:
                    check("seb_peer_close", lib().seb_peer_close(p))
            dist.barrier(group=self.group)  # every peer closed its mapping of this rank's region
        with torch.cuda.device(self.device):
            for p in self._owned:
                check("seb_peer_free", lib().seb_peer_free(p))
        self._closed = True
