"""Multi-GPU partitioning of the i2_s path: N-split GEMM with the output gather fused into the epilogue,
and data-parallel sharding of independent observations.

N-split (very large M, e.g. 16384 tokens): rank r of g owns weight rows [n0_r, n1_r) (b2s_nsplit_range) --
a contiguous byte range of the i2_s tensor, cut out with its fp32 scale by b2s_i2s_shard_rows. The
activations are replicated (every rank quantizes the full X). Each rank's GEMM epilogue writes its column
slice straight into the root GPU's output buffer over NVLink: the root exports the buffer
(b2s_peer_export), the 72 handle bytes are broadcast through the process group (transport only), every
other rank maps it (b2s_peer_open) and passes `root_ptr + n0_r` with row stride N as the kernel's output
(plain peer stores; no multicast, no separate gather kernel or collective). A process-group barrier after
the ranks' streams complete makes the gathered Y readable on the root.

Data parallel (independent observations): rank r takes a contiguous slice of the observation list; no
data-path collective.
"""
from __future__ import annotations

import ctypes as C


def row_ranges(n_rows: int, world: int) -> list[tuple[int, int]]:
    """Balanced contiguous ranges [n0, n1) covering n_rows over `world` ranks (the library's split)."""
    import b2s
    if world <= 0 or n_rows < 0:
        raise ValueError("world must be positive and n_rows non-negative")
    return [b2s.nsplit_range(n_rows, world, r) for r in range(world)]


def shard_range(n_items: int, rank: int, world: int) -> tuple[int, int]:
    """Data-parallel slice [i0, i1) of n_items for `rank`."""
    return row_ranges(n_items, world)[rank]


def shard_i2s_rows(packed, n_rows: int, k: int, n0: int, n1: int, rowpadded: bool = False):
    """The i2_s bytes of weight rows [n0, n1) as a standalone i2_s tensor (codes + 32-byte scale trailer)."""
    import b2s
    return b2s.i2s_shard_rows(packed, n_rows, k, n0, n1, rowpadded=rowpadded)


class PeerBuffer:
    """A device buffer allocated on the root rank and mapped into every rank through the library's
    b2s_peer_export / b2s_peer_open.

    `ptr` is this rank's device address of the buffer (the root's own allocation on the root, the opened
    mapping elsewhere). `tensor` is a torch view on the root. Collective: every rank of `group` must
    construct it, in the same order.
    """

    def __init__(self, nbytes: int, group=None, root: int = 0):
        import torch
        import torch.distributed as dist
        import b2s

        self._b2s = b2s
        self.nbytes = int(nbytes)
        self.root = root
        self.rank = dist.get_rank(group)
        self._owned = None
        self._opened = None
        payload = [None]
        if self.rank == root:
            self._owned = torch.empty(self.nbytes, dtype=torch.uint8, device="cuda")
            payload = [b2s.peer_export(self._owned.data_ptr())]
        dist.broadcast_object_list(payload, src=root, group=group)
        if self.rank == root:
            self.ptr = int(self._owned.data_ptr())
        else:
            self._opened = b2s.peer_open(payload[0])
            self.ptr = self._opened

    def tensor(self, shape, dtype):
        """Torch view of the root's buffer (no copy); valid on the root only."""
        if self._owned is None:
            raise ValueError("only the root holds a torch view of the buffer")
        n = 1
        for d in shape:
            n *= int(d)
        return self._owned.view(dtype)[:n].view(*shape)

    def close(self):
        if self._opened is not None:
            self._b2s.peer_close(self._opened)
            self._opened = None
        self._owned = None


def nsplit_mul_mat_q8(b2s_mod, W_local, q, s, sums, M: int, y_ptr: int, ldy: int, n0: int, stream=None) -> None:
    """Runs this rank's N-slice of the MUL_MAT, writing columns [n0, n0 + n_local) of the [M, ldy] fp32
    output at device address y_ptr (a peer mapping of the root's buffer, or a local one)."""
    lib = b2s_mod.lib()
    out = int(y_ptr) + 4 * int(n0)
    b2s_mod.check(lib.b2s_mul_mat_q8_ex(C.byref(W_local), q.data_ptr(), q.stride(0), s.data_ptr(), sums.data_ptr(),
                                        int(M), out, int(ldy), 0, b2s_mod._stream(stream)))
