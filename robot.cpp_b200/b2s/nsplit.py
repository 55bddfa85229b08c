"""Multi-GPU partitioning of the i2_s path: N-split GEMM with the output gather fused into the epilogue,
and data-parallel sharding of independent observations.

N-split (very large M, e.g. 16384 tokens): rank r of g owns weight rows [n0_r, n1_r) -- a contiguous byte
range of the i2_s tensor when K % 128 == 0 (rows are K/4 bytes each), re-wrapped with the tensor's
fp32 scale as a standalone i2_s tensor. The activations are replicated (every rank quantizes the full X).
Each rank's GEMM epilogue writes its column slice straight into the root GPU's output buffer over
NVLink: the buffer is cudaMalloc'd on the root, its CUDA IPC handle is broadcast through the process
group, and every rank passes `root_ptr + n0_r` with row stride N as the kernel's output (plain peer
stores; no multicast, no separate gather kernel or collective). A process-group barrier after the
ranks' streams complete makes the gathered Y readable on the root.

Data parallel (independent observations): rank r takes a contiguous slice of the observation list; no
data-path collective.
"""
from __future__ import annotations

import numpy as np


def row_ranges(n_rows: int, world: int) -> list[tuple[int, int]]:
    """Balanced contiguous ranges [n0, n1) covering n_rows over `world` ranks (sizes differ by <= 1)."""
    if world <= 0 or n_rows < 0:
        raise ValueError("world must be positive and n_rows non-negative")
    base, extra = divmod(n_rows, world)
    out, n0 = [], 0
    for r in range(world):
        n1 = n0 + base + (1 if r < extra else 0)
        out.append((n0, n1))
        n0 = n1
    return out


def shard_range(n_items: int, rank: int, world: int) -> tuple[int, int]:
    """Data-parallel slice [i0, i1) of n_items for `rank`."""
    return row_ranges(n_items, world)[rank]


def shard_i2s_rows(packed: np.ndarray, n_rows: int, k: int, n0: int, n1: int) -> np.ndarray:
    """The i2_s bytes of weight rows [n0, n1) as a standalone i2_s tensor (codes + 32-byte scale trailer).

    Needs K % 128 == 0 so that every row is its own run of K/4 bytes in the flattened layout (other K are
    row-padded first with b2s_i2s_repack_rows / the oracle's to_rowpadded and sharded with K rounded up).
    """
    if k % 128 != 0:
        raise ValueError("row sharding of flattened i2_s needs K % 128 == 0; repack rows first")
    if not (0 <= n0 <= n1 <= n_rows):
        raise ValueError("bad row range")
    packed = np.asarray(packed, dtype=np.uint8)
    rb = k // 4
    code_bytes = n_rows * rb
    if packed.size != code_bytes + 32:
        raise ValueError("packed buffer size does not match N*K/4 + 32")
    out = np.empty((n1 - n0) * rb + 32, np.uint8)
    out[: (n1 - n0) * rb] = packed[n0 * rb: n1 * rb]
    out[(n1 - n0) * rb:] = packed[code_bytes: code_bytes + 32]
    return out


class PeerBuffer:
    """A device buffer allocated on the root rank and mapped into every rank through CUDA IPC.

    `ptr` is this rank's device address of the buffer (the root's own allocation on the root, the opened
    IPC mapping elsewhere). `tensor()` gives a torch view on the root. Collective: every rank of `group`
    must construct it, in the same order.
    """

    def __init__(self, nbytes: int, group=None, root: int = 0):
        import torch
        import torch.distributed as dist
        from cuda.bindings import runtime as rt

        self._rt = rt
        self.nbytes = int(nbytes)
        self.root = root
        self.rank = dist.get_rank(group)
        self._owned = None
        self._opened = None
        payload = [None]
        if self.rank == root:
            err, ptr = rt.cudaMalloc(self.nbytes)
            _check(err, "cudaMalloc")
            self._owned = int(ptr)
            err, handle = rt.cudaIpcGetMemHandle(self._owned)
            _check(err, "cudaIpcGetMemHandle")
            payload = [bytes(handle.reserved)]
        dist.broadcast_object_list(payload, src=root, group=group)
        if self.rank == root:
            self.ptr = self._owned
        else:
            handle = rt.cudaIpcMemHandle_t()
            handle.reserved = payload[0]
            err, ptr = rt.cudaIpcOpenMemHandle(handle, rt.cudaIpcMemLazyEnablePeerAccess)
            _check(err, "cudaIpcOpenMemHandle")
            self._opened = int(ptr)
            self.ptr = self._opened
        self._torch = torch

    def tensor(self, shape, dtype):
        """Torch view of the buffer (no copy); valid on any rank, meaningful to read on the root."""
        torch = self._torch
        itemsize = torch.empty((), dtype=dtype).element_size()
        n = int(np.prod(shape))
        if n * itemsize > self.nbytes:
            raise ValueError("view larger than the buffer")

        class _Cai:
            pass
        obj = _Cai()
        typestr = {torch.float32: "<f4", torch.int32: "<i4", torch.uint8: "|u1", torch.int8: "|i1"}[dtype]
        obj.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (self.ptr, False),
                                        "version": 3, "strides": None}
        return torch.as_tensor(obj, device=torch.device("cuda", torch.cuda.current_device()))

    def close(self):
        rt = self._rt
        if self._opened is not None:
            rt.cudaIpcCloseMemHandle(self._opened)
            self._opened = None
        if self._owned is not None:
            rt.cudaFree(self._owned)
            self._owned = None


def _check(err, what):
    from cuda.bindings import runtime as rt
    if err != rt.cudaError_t.cudaSuccess:
        raise RuntimeError(f"{what} failed: {err}")


def nsplit_mul_mat_q8(b2s_mod, W_local, q, s, sums, M: int, y_ptr: int, ldy: int, n0: int, stream=None) -> None:
    """Runs this rank's N-slice of the MUL_MAT, writing columns [n0, n0 + n_local) of the [M, ldy] fp32
    output at device address y_ptr (a peer mapping of the root's buffer, or a local one)."""
    import ctypes as C
    lib = b2s_mod.lib()
    out = int(y_ptr) + 4 * int(n0)
    b2s_mod.check(lib.b2s_mul_mat_q8_ex(C.byref(W_local), q.data_ptr(), q.stride(0), s.data_ptr(), sums.data_ptr(),
                                        int(M), out, int(ldy), 0, b2s_mod._stream(stream)))
