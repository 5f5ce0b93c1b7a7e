"""KV-head-sharded decode fused with the all-gather of its output, over NVLink peer memory.

Rank r of N runs K2 for its KV heads and writes its attention-output rows straight into every
rank's full output buffer ``[B, N * Hq/N, D]`` (``ts_paged_decode_peer``): the all-gather is the
kernel's own stores over NVLink, so there is no collective kernel to schedule beside a decode
kernel that occupies every SM. The grid's last CTA then publishes the call's epoch into every
rank's signal array, and ``ts_wait_peers`` (one small kernel on the consumer's stream) waits with
a bounded spin until all ranks have published it.

The buffers are plain device allocations (``ts_peer_alloc``) shared between the ranks'
processes with CUDA IPC handles, exchanged once over ``torch.distributed``.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from tokenserve_b200 import ops


class _DeviceArray:
    """A torch view of raw device memory (``__cuda_array_interface__``)."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str) -> None:
        self.__cuda_array_interface__ = {
            "data": (ptr, False), "shape": shape, "typestr": typestr, "version": 3,
        }  # fmt: skip


_TYPESTR = {torch.bfloat16: "<V2", torch.float16: "<f2", torch.int32: "<i4"}


def _view(ptr: int, shape: tuple[int, ...], dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    if dtype == torch.bfloat16:  # no numpy typestr for bf16: view 16-bit words
        t = torch.as_tensor(_DeviceArray(ptr, shape, "<i2"), device=device)
        return t.view(torch.bfloat16)
    return torch.as_tensor(_DeviceArray(ptr, shape, _TYPESTR[dtype]), device=device)


class PeerGather:
    """``nbuf`` full output buffers and one signal array per rank, mapped on every rank.

    ``decode(p, ...)`` runs this rank's fused decode into buffer ``p`` of every rank and returns
    its epoch; ``wait(epoch)`` enqueues the wait for all ranks' writes of that epoch on the
    current stream; ``full[p]`` is this rank's buffer ``p`` as a tensor ``[B, N * Hq_r, D]``.
    """

    def __init__(self, batch: int, q_heads_per_rank: int, head_dim: int, dtype: torch.dtype,
                 nbuf: int = 4, group: dist.ProcessGroup | None = None) -> None:  # fmt: skip
        self.lib = ops.load_library()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.group = group
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.shape = (batch, self.world * q_heads_per_rank, head_dim)
        self.dtype = dtype
        nbytes = batch * self.world * q_heads_per_rank * head_dim * torch.finfo(dtype).bits // 8
        self._own: list[int] = []
        for _ in range(nbuf):
            self._own.append(self._alloc(nbytes))
        self._own.append(self._alloc(4 * self.world))  # signal array
        self.full = [_view(p, self.shape, dtype, self.device) for p in self._own[:nbuf]]
        self.signals = _view(self._own[-1], (self.world,), torch.int32, self.device)
        self.signals.zero_()
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize()
        # Exchange the handles and map every peer's buffers.
        handles = []
        for p in self._own:
            h = ctypes.create_string_buffer(64)
            ops._check(self.lib.ts_ipc_get_handle(p, ctypes.cast(h, ctypes.c_void_p)),
                       "ipc_get_handle")  # fmt: skip
            handles.append(h.raw)
        everyone: list = [None] * self.world
        dist.all_gather_object(everyone, handles, group=group)
        self._opened: list[int] = []
        ptrs = []  # ptrs[r][i]: rank r's buffer i as mapped here
        for r in range(self.world):
            if r == self.rank:
                ptrs.append(list(self._own))
                continue
            row = []
            for h in everyone[r]:
                out = ctypes.c_void_p()
                hb = ctypes.create_string_buffer(h, 64)
                ops._check(self.lib.ts_ipc_open(ctypes.cast(hb, ctypes.c_void_p), ctypes.byref(out)),
                           "ipc_open")  # fmt: skip
                self._opened.append(out.value)
                row.append(out.value)
            ptrs.append(row)
        self.dst = [torch.tensor([ptrs[r][i] for r in range(self.world)], dtype=torch.int64,
                                 device=self.device) for i in range(nbuf)]  # fmt: skip
        self.sig = torch.tensor([ptrs[r][nbuf] for r in range(self.world)], dtype=torch.int64,
                                device=self.device)  # fmt: skip
        self.epoch = 0
        dist.barrier(group=group)

    def _alloc(self, nbytes: int) -> int:
        out = ctypes.c_void_p()
        ops._check(self.lib.ts_peer_alloc(nbytes, ctypes.byref(out)), "peer_alloc")
        return int(out.value)

    def decode(self, p: int, query: torch.Tensor, key_pool: torch.Tensor, value_pool: torch.Tensor,
               block_tables: torch.Tensor, context_lens: torch.Tensor, scale: float,
               workspace: torch.Tensor, reuse_plan: bool = False, pull: bool = False) -> int:  # fmt: skip
        """This rank's decode into buffer ``p``: its rows stored into every rank's buffer
        (``pull=False``, then :meth:`wait`) or into its own only (``pull=True``, then
        :meth:`gather`, which fetches the other ranks' rows). Returns the call's epoch."""
        nb, hkv, bs, d = ops._pool_dims(key_pool)
        hq = query.shape[1]
        qs = ops._rows(query, hq, d, "query")
        self.epoch += 1
        ws_bytes = workspace.numel() * workspace.element_size()
        fn = self.lib.ts_paged_decode_publish if pull else self.lib.ts_paged_decode_peer
        code = fn(
            ops._ptr(self.dst[p]), self.world, self.rank, ops._ptr(self.sig), self.epoch,
            ops._ptr(query), qs, ops._ptr(key_pool), ops._ptr(value_pool),
            ops._ptr(block_tables), block_tables.shape[1], ops._ptr(context_lens),
            query.shape[0], hq, hkv, d, bs, nb, float(scale), ops._dtype(key_pool),
            ops._ptr(workspace), ws_bytes, int(reuse_plan), ops._stream(),
        )  # fmt: skip
        ops._check(code, "paged_decode_peer")
        return self.epoch

    def gather(self, p: int, epoch: int) -> None:
        """Enqueues, on the current stream, the wait for every rank's ``epoch`` and the copy of
        their rows into this rank's buffer ``p`` (the pull form of the exchange)."""
        b, h, d = self.shape
        code = self.lib.ts_gather_peers(ops._ptr(self.dst[p]), self.world, self.rank,
                                        ops._ptr(self.signals), epoch, b, h // self.world, d,
                                        ops.DTYPE_CODES[self.dtype], ops._ptr(self.status),
                                        ops._stream())  # fmt: skip
        ops._check(code, "gather_peers")

    def wait(self, epoch: int) -> None:
        code = self.lib.ts_wait_peers(ops._ptr(self.signals), self.world, epoch,
                                      ops._ptr(self.status), ops._stream())  # fmt: skip
        ops._check(code, "wait_peers")

    def check(self) -> None:
        """Raises if any wait since the last check timed out (a rank that never published its
        epoch); the status word is cleared either way, so one timeout is reported once."""
        code = int(self.status.item())
        if code:
            self.status.zero_()
            raise ops.KernelError("wait_peers: a rank did not publish its output in time")

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's; every rank must be done with them."""
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for p in self._opened:
            self.lib.ts_ipc_close(p)
        self._opened = []
        dist.barrier(group=self.group)
        for p in self._own:
            self.lib.ts_peer_free(p)
        self._own = []
