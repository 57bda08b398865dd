"""N-split of the GEMM across the GPUs of one node (one process per GPU).

Rank r owns columns ``[col_begin(N, P, r), col_begin(N, P, r+1))`` of B and C
(rows of B_q for the K-packed INT4 layout); A is replicated. Each rank runs the
single-GPU kernel on its shard; with ``replicate_C`` the shards are all-gathered
over NCCL (NVLink) into the full row-major C on every rank. A C registered with
``register_output`` (a collective that maps it into every rank through CUDA IPC)
is instead filled by the GEMM's own epilogue (fp16, INT8 row/col, INT4), which stores each
finished tile into every rank's copy over NVLink. A C from ``multicast_output`` (CUDA
symmetric memory bound to one NVLink multicast object) takes the same route with one
multicast store per tile, which the NVSwitch fabric delivers to every rank. The NCCL
communicator belongs to the C library; its unique id is exchanged through the
torch.distributed store of the already-initialised process group.
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import check, lib
from .api import _need, _ptr, _stream


def col_begin(N: int, nranks: int, rank: int) -> int:
    """First column owned by ``rank`` (first N % P ranks own one extra column)."""
    return lib().clove_nsplit_col_begin(int(N), int(nranks), int(rank))


class NSplit:
    """NCCL context of the N-split. Create on every rank after torch.distributed init."""

    def __init__(self, rank: int, nranks: int, store=None, tag: str = "clove_nsplit"):
        import torch.distributed as dist
        self.rank, self.nranks = int(rank), int(nranks)
        uid = (ctypes.c_uint8 * 128)()
        if store is None:
            store = dist.distributed_c10d._get_default_store()
        if self.rank == 0:
            check(lib().clove_nsplit_get_unique_id(uid))
            store.set(tag, bytes(uid))
        else:
            data = store.get(tag)
            ctypes.memmove(uid, data, 128)
        ctx = ctypes.c_void_p()
        check(lib().clove_nsplit_init(ctypes.byref(ctx), self.nranks, self.rank, uid))
        self._ctx = ctx
        self._outputs = {}

    def close(self) -> None:
        if getattr(self, "_ctx", None) is not None and self._ctx.value:
            check(lib().clove_nsplit_destroy(self._ctx))
            self._ctx = None
            self._outputs = {}

    def register_output(self, C_full: torch.Tensor) -> None:
        """Collective: every rank registers its own [M, N] fp16 replicated output in
        the same order; gemm_fp16(..., C_full=C_full, replicate_C=True) then writes
        every rank's copy from the GEMM epilogue (no all-gather)."""
        # A rank whose argument is bad still takes part (with a null pointer, which
        # fails the registration on every rank) so that no rank waits alone.
        err, ptr, nbytes = None, None, 0
        try:
            _need(C_full, "C_full", torch.float16, 2)
            ptr, nbytes = _ptr(C_full), C_full.numel() * C_full.element_size()
        except Exception as e:  # raised after the collective call
            err = e
        rc = lib().clove_nsplit_register_output(self._ctx, ptr, nbytes)
        if err is not None:
            raise err
        check(rc)
        self._outputs[C_full.data_ptr()] = C_full  # keeps the memory alive while mapped

    def multicast_output(self, M: int, N: int, group=None) -> torch.Tensor:
        """Collective: an [M, N] fp16 replicated output in CUDA symmetric memory, every
        rank's copy bound to one NVLink multicast object, registered for the
        replicated route (each finished tile then leaves once, as multicast stores).
        Raises on every rank when any rank's GPU offers no multicast. Release with
        ``unregister_output`` on every rank."""
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem
        g = group if group is not None else dist.group.WORLD
        C = symm_mem.empty((int(M), int(N)), dtype=torch.float16,
                           device=torch.device("cuda", torch.cuda.current_device()))
        handle = symm_mem.rendezvous(C, g)
        mc = int(getattr(handle, "multicast_ptr", 0) or 0)
        # Every rank calls the registration (a rank without multicast passes NULL,
        # which fails it on every rank) so that no rank waits alone.
        rc = lib().clove_nsplit_register_output_multicast(
            self._ctx, C.data_ptr(), mc if mc else None, C.numel() * C.element_size())
        if rc != 0:
            del handle, C
            check(rc)
        self._outputs[C.data_ptr()] = (C, handle)  # keeps memory and binding alive
        return C

    def unregister_output(self, C_full: torch.Tensor) -> None:
        """Collective: unmaps C_full on every rank."""
        try:
            ptr = _ptr(C_full)
        except Exception:
            ptr = None  # still takes part; fails on every rank
        check(lib().clove_nsplit_unregister_output(self._ctx, ptr))
        self._outputs.pop(C_full.data_ptr(), None)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def cols(self, N: int) -> tuple[int, int]:
        return col_begin(N, self.nranks, self.rank), col_begin(N, self.nranks, self.rank + 1)

    def gemm_fp16(self, A, B_shard, N, C_shard=None, C_full=None, alpha=1.0,
                  replicate_C=False, stream=None):
        _need(A, "A", torch.float16, 2)
        _need(B_shard, "B_shard", torch.float16, 2)
        M, K = A.shape
        c0, c1 = self.cols(N)
        if C_shard is None:
            C_shard = torch.empty((M, c1 - c0), dtype=torch.float16, device=A.device)
        if replicate_C and C_full is None:
            C_full = torch.empty((M, N), dtype=torch.float16, device=A.device)
        check(lib().clove_nsplit_gemm_fp16(self._ctx, _ptr(A), _ptr(B_shard), _ptr(C_shard),
                                           _ptr(C_full) if C_full is not None else None, M, N, K,
                                           float(alpha), int(bool(replicate_C)), _stream(stream)))
        return C_full if replicate_C else C_shard

    def gemm_int4(self, A_q, A_scale, A_zero, B_q_shard, B_scale_shard, B_zero_shard, N,
                  C_shard=None, C_full=None, replicate_C=False, stream=None):
        M, K = A_q.shape[0], 2 * A_q.shape[1]
        c0, c1 = self.cols(N)
        if C_shard is None:
            C_shard = torch.empty((M, c1 - c0), dtype=torch.float16, device=A_q.device)
        if replicate_C and C_full is None:
            C_full = torch.empty((M, N), dtype=torch.float16, device=A_q.device)
        check(lib().clove_nsplit_gemm_int4(
            self._ctx, _ptr(A_q), _ptr(A_scale), _ptr(A_zero), _ptr(B_q_shard), _ptr(B_scale_shard),
            _ptr(B_zero_shard), _ptr(C_shard), _ptr(C_full) if C_full is not None else None,
            M, N, K, int(bool(replicate_C)), _stream(stream)))
        return C_full if replicate_C else C_shard

    def gemm_int8_rowcol(self, A_q, B_q_shard, A_row_scale, B_col_scale_shard, N, C_shard=None,
                         C_full=None, replicate_C=False, stream=None):
        M, K = A_q.shape
        c0, c1 = self.cols(N)
        if C_shard is None:
            C_shard = torch.empty((M, c1 - c0), dtype=torch.float16, device=A_q.device)
        if replicate_C and C_full is None:
            C_full = torch.empty((M, N), dtype=torch.float16, device=A_q.device)
        check(lib().clove_nsplit_gemm_int8_rowcol(
            self._ctx, _ptr(A_q), _ptr(B_q_shard), _ptr(A_row_scale), _ptr(B_col_scale_shard),
            _ptr(C_shard), _ptr(C_full) if C_full is not None else None, M, N, K,
            int(bool(replicate_C)), _stream(stream)))
        return C_full if replicate_C else C_shard
