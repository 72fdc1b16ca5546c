"""Multi-device paged MLA: request sharding and the cross-device KV split of long contexts.

Two strategies, one process per GPU:
  - request sharding (``inputs.shard``): whole sequences are assigned to devices by token count;
    each device owns the pages of its sequences and runs the kernel on them; no collective is
    on the data path.
  - context split (``context_split`` + ``context_merge``): for very long single-token decodes,
    every device holds a contiguous, page-aligned range of each sequence's positions and
    computes a partial result (f32 output normalised over its range, natural-log lse); the
    library's ``tq_mla_context_merge`` all-gathers the partials over its own NCCL communicator
    and merges them by log-sum-exp on every device. The reference plans this as decode context
    parallelism (docs/ARCHITECTURE.md:240-241,313) behind a per-worker ``Comm``
    (docs/ARCHITECTURE.md:136-137, lifecycle :242-254).
Python only sets things up: it carries the communicator's 128-byte id from rank 0 to the other
ranks (any ``torch.distributed`` group, gloo included) and holds the device buffers; the
collective and the merge run in libtq_mla.so.
"""

import ctypes

import numpy as np

from . import inputs

PAGE_ROWS = 64


def context_ranges(kv_len, world):
    """Page-aligned position ranges ``[(start, end)] * world`` for one sequence of ``kv_len``."""
    pages = (int(kv_len) + PAGE_ROWS - 1) // PAGE_ROWS
    cuts = [(pages * r) // world for r in range(world + 1)]
    return [(min(kv_len, cuts[r] * PAGE_ROWS), min(kv_len, cuts[r + 1] * PAGE_ROWS))
            for r in range(world)]


def context_split(w: inputs.Workload, world: int, rank: int) -> inputs.Workload:
    """This device's share of a single-token decode batch: positions ``[a_r, b_r)`` of each
    sequence, as sequences of their own (cache contents keep their global data offsets)."""
    if (w.q_per_seq != 1).any():
        raise ValueError("the context split applies to single-token decode")
    if ((w.prefix + 1) < w.kv_len).any():
        raise ValueError("the context split needs every cached position to be visible")
    starts, lens = [], []
    for n in w.kv_len:
        a, b = context_ranges(int(n), world)[rank]
        starts.append(a)
        lens.append(b - a)
    starts = np.asarray(starts, dtype=np.int64)
    lens = np.asarray(lens, dtype=np.int64)
    tok_off = np.concatenate([[0], np.cumsum(w.kv_len)[:-1]]).astype(np.int64) + starts
    sub = inputs.Workload(f"{w.name} context part {rank}/{world}", w.seed, w.heads, w.width, lens,
                          w.q_per_seq.copy(), lens - 1, w.scale,
                          seq_global=np.arange(w.sequences),
                          token_global=np.arange(w.sequences, dtype=np.int64),
                          tok_off_global=tok_off)
    return inputs._finish(sub)


class Comm:
    """This rank's communicator (``tq_comm_*``): an NCCL communicator over the GPUs of the job.

    Created collectively by every rank with its GPU current. A communicator whose collective
    failed (``TqError`` with status 106) must be aborted (``abort``) and never reused.
    """

    def __init__(self, comm_id: bytes, world: int, rank: int):
        from . import _abi

        cid = _abi.TqCommId()
        ctypes.memmove(ctypes.addressof(cid), comm_id, 128)
        handle = ctypes.c_void_p()
        _abi.raise_for(_abi.lib.tq_comm_init(ctypes.byref(cid), world, rank, ctypes.byref(handle)))
        self.handle, self.world, self.rank = handle, world, rank
        self._gather = {}

    @staticmethod
    def new_id() -> bytes:
        from . import _abi

        cid = _abi.TqCommId()
        _abi.raise_for(_abi.lib.tq_comm_unique_id(ctypes.byref(cid)))
        return ctypes.string_at(ctypes.addressof(cid), 128)

    @classmethod
    def from_process_group(cls, group=None):
        """All ranks of ``group`` call this; rank 0's id reaches the others through the group."""
        import torch.distributed as dist

        rank, world = dist.get_rank(group), dist.get_world_size(group)
        box = [cls.new_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0, group=group)
        return cls(box[0], world, rank)

    def destroy(self):
        from . import _abi

        if self.handle:
            self._gather.clear()
            st = _abi.lib.tq_comm_destroy(self.handle)
            self.handle = None
            _abi.raise_for(st)

    def abort(self):
        from . import _abi

        if self.handle:
            self._gather.clear()
            st = _abi.lib.tq_comm_abort(self.handle)
            self.handle = None
            _abi.raise_for(st)

    def gather_buffers(self, tokens, heads, device):
        import torch

        key = (tokens, heads, str(device))
        if key not in self._gather:
            self._gather[key] = (
                torch.empty((self.world, tokens, heads, 512), dtype=torch.float32, device=device),
                torch.empty((self.world, tokens, heads), dtype=torch.float32, device=device))
        return self._gather[key]


def context_merge(comm: Comm, part_out, part_lse, out=None, lse=None, stream=None):
    """Merge this rank's partial (``f32 [T,H,512]``, ``f32 [T,H]``) with every other rank's:
    returns ``(out [T,H,512], lse [T,H])``, identical on all ranks. One call of
    ``tq_mla_context_merge`` (NCCL all-gather, then the LSE merge kernel) on ``stream``."""
    import torch

    from . import _abi
    from .ops import _TORCH_DTYPE, _stream_handle

    t, h, d = part_out.shape
    if d != 512 or part_out.dtype != torch.float32 or part_lse.shape != (t, h):
        raise ValueError("partials must be f32 [T, H, 512] and f32 [T, H]")
    part_out, part_lse = part_out.contiguous(), part_lse.contiguous()
    if out is None:
        out = torch.empty((t, h, 512), dtype=torch.bfloat16, device=part_out.device)
    if lse is None:
        lse = torch.empty((t, h), dtype=torch.float32, device=part_out.device)
    g_out, g_lse = comm.gather_buffers(t, h, part_out.device)
    p = _abi.TqContextMergeParams()
    p.tokens, p.heads = t, h
    p.part_out, p.part_lse = part_out.data_ptr(), part_lse.data_ptr()
    p.gather_out, p.gather_lse = g_out.data_ptr(), g_lse.data_ptr()
    p.gather_out_bytes = g_out.numel() * 4
    p.gather_lse_bytes = g_lse.numel() * 4
    p.out, p.lse = out.data_ptr(), lse.data_ptr()
    p.out_stride_token = out.stride(0) * out.element_size()
    p.out_stride_head = out.stride(1) * out.element_size()
    p.out_dtype = _TORCH_DTYPE[out.dtype]
    _abi.raise_for(_abi.lib.tq_mla_context_merge(ctypes.byref(p), comm.handle,
                                                 _stream_handle(stream)))
    return out, lse


class _DeviceArray:
    """Exposes a device address range to torch (``__cuda_array_interface__``, no copy)."""

    def __init__(self, address, shape, typestr):
        self.__cuda_array_interface__ = {"data": (int(address), False), "shape": tuple(shape),
                                         "typestr": typestr, "version": 3}


class PeerMerge:
    """The context merge over NVLink peer memory (``tq_peer_merge_*``): created collectively on
    ``comm`` for ``tokens`` x ``heads`` rows. ``part_out`` (f32 ``[T, H, 512]``) and ``part_lse``
    (f32 ``[T, H]``) view this rank's exchange region: decode into them, then call ``merge``.
    Every rank calls ``merge`` once per step, in the same order."""

    def __init__(self, comm: Comm, tokens: int, heads: int):
        import torch

        from . import _abi

        self.comm = comm
        self.handle = ctypes.c_void_p()
        _abi.raise_for(_abi.lib.tq_peer_merge_create(comm.handle, tokens, heads,
                                                     ctypes.byref(self.handle)))
        po, pl = ctypes.c_uint64(), ctypes.c_uint64()
        _abi.raise_for(_abi.lib.tq_peer_merge_partials(self.handle, ctypes.byref(po),
                                                       ctypes.byref(pl)))
        self.part_out = torch.as_tensor(_DeviceArray(po.value, (tokens, heads, 512), "<f4"),
                                        device="cuda")
        self.part_lse = torch.as_tensor(_DeviceArray(pl.value, (tokens, heads), "<f4"),
                                        device="cuda")

    def merge(self, out, lse, stream=None):
        """The merged ``out`` (bf16 or f32 ``[T, H, 512]``) and ``lse`` (f32 ``[T, H]``)."""
        from . import _abi
        from .ops import _TORCH_DTYPE, _stream_handle

        _abi.raise_for(_abi.lib.tq_peer_merge(
            self.handle, out.data_ptr(), lse.data_ptr(), out.stride(0) * out.element_size(),
            out.stride(1) * out.element_size(), _TORCH_DTYPE[out.dtype], _stream_handle(stream)))
        return out, lse

    def device_error(self, stream=None):
        from . import _abi
        from .ops import _stream_handle

        flags = ctypes.c_int32()
        _abi.raise_for(_abi.lib.tq_peer_merge_read_error(self.handle, _stream_handle(stream),
                                                         ctypes.byref(flags)))
        return flags.value

    def destroy(self):
        from . import _abi

        if self.handle:
            self.part_out = self.part_lse = None
            _abi.raise_for(_abi.lib.tq_peer_merge_destroy(self.handle))
            self.handle = ctypes.c_void_p()
