"""Host mirror of the reference's SMLA operator interface over the native C ABI.

``validate`` mirrors ``SmlaParams::new`` (crates/tq-core/src/contracts.rs:437-493) and raises
``ContractError(field, kind)`` with the same field names and violation kinds. ``MlaLaunch`` is
the validated launch (the planned ``sparse_mla_decode`` launcher of docs/ARCHITECTURE.md:111-113,
in dense paged form): it owns nothing but a workspace, and every launch goes through
``tq_mla_decode`` / ``tq_mla_prefill`` in libtq_mla.so. Torch is used only to hold device memory
and to name the current stream.
"""

import ctypes
import math

import torch

from . import _abi
from ._abi import ContractError, TqError, lib, raise_for  # noqa: F401  (re-exported)

_TORCH_DTYPE = {
    torch.bfloat16: _abi.DTYPE_BF16,
    torch.int32: _abi.DTYPE_I32,
    torch.float32: _abi.DTYPE_F32,
    torch.uint8: _abi.DTYPE_U8,
}
PAYLOAD = {_abi.KV_BF16: 1024, _abi.KV_FP8_E4M3: 528, _abi.KV_BF16_ROPE576: 1152}


def tensor_spec(shape, strides_bytes, dtype, address, buffer_bytes):
    t = _abi.TqTensorSpec()
    t.rank = len(shape)
    for i, (d, s) in enumerate(zip(shape, strides_bytes)):
        t.shape[i] = int(d)
        t.strides_bytes[i] = int(s)
    t.dtype = int(dtype)
    t.device_address = int(address)
    t.buffer_bytes = int(buffer_bytes)
    return t


def _capacity(t: torch.Tensor) -> int:
    return t.untyped_storage().nbytes() - t.storage_offset() * t.element_size()


def spec_of(t: torch.Tensor):
    """Declaration of a torch tensor: its shape, byte strides, address and reachable bytes."""
    es = t.element_size()
    return tensor_spec(t.shape, [s * es for s in t.stride()], _TORCH_DTYPE[t.dtype],
                       t.data_ptr(), _capacity(t))


def pool_spec(kv: torch.Tensor, kv_format: int):
    """The paged pool as ``u8 [P, 64, payload]`` with strides ``[64 r, r, 1]``.

    ``kv`` is ``[P, 64, W]`` of any element type whose rows are contiguous (``W * itemsize``
    bytes of payload per row, row stride ``r = kv.stride(1) * itemsize``).
    """
    es = kv.element_size()
    payload = PAYLOAD[kv_format]
    return tensor_spec([kv.shape[0], kv.shape[1], payload],
                       [kv.stride(0) * es, kv.stride(1) * es, 1], _abi.DTYPE_U8,
                       kv.data_ptr(), _capacity(kv))


def make_spec(q, kv, page_table, seq_id, q_pos, kv_len, out, lse, *, scale, kv_format=None):
    if kv_format is None:
        kv_format = _abi.KV_BF16_ROPE576 if q.shape[-1] == 576 else _abi.KV_BF16
    s = _abi.TqMlaSpec()
    s.q = spec_of(q)
    s.kv = pool_spec(kv, kv_format)
    s.page_table = spec_of(page_table)
    s.seq_id = spec_of(seq_id)
    s.q_pos = spec_of(q_pos)
    s.kv_len = spec_of(kv_len)
    s.out = spec_of(out)
    s.lse = spec_of(lse)
    s.kv_format = kv_format
    s.softmax_scale = float(scale)
    return s


def validate(spec, query_counts, *, prefill=False, idx=None, k_len=None):
    """Validate ``spec`` against the host plan; returns ``TqMlaParams`` or raises.

    With ``idx`` / ``k_len`` (tensor declarations, ``TqTensorSpec``) the plan is a sparse top-k
    decode plan (``tq_mla_sparse_validate``).
    """
    params = _abi.TqMlaParams()
    err = _abi.TqContractError()
    counts = list(int(c) for c in query_counts)
    if idx is not None:
        if any(c < 0 or c > 255 for c in counts):
            raise ContractError("query_counts", 9)
        arr = (ctypes.c_uint8 * max(1, len(counts)))(*counts)
        st = lib.tq_mla_sparse_validate(ctypes.byref(spec), ctypes.byref(idx), ctypes.byref(k_len),
                                        arr, len(counts), ctypes.byref(params), ctypes.byref(err))
        raise_for(st, err)
        return params
    if prefill:
        arr = (ctypes.c_uint32 * max(1, len(counts)))(*counts)
        st = lib.tq_mla_prefill_validate(ctypes.byref(spec), arr, len(counts),
                                         ctypes.byref(params), ctypes.byref(err))
    else:
        if any(c < 0 or c > 255 for c in counts):
            raise ContractError("query_counts", 9)
        arr = (ctypes.c_uint8 * max(1, len(counts)))(*counts)
        st = lib.tq_mla_validate(ctypes.byref(spec), arr, len(counts), ctypes.byref(params),
                                 ctypes.byref(err))
    raise_for(st, err)
    return params


def workspace_bytes(params, device=None):
    dev = torch.cuda.current_device() if device is None else int(device)
    n = ctypes.c_uint64()
    raise_for(lib.tq_mla_workspace_bytes(ctypes.byref(params), dev, ctypes.byref(n)))
    return n.value


def workspace_layout(params, device=None):
    dev = torch.cuda.current_device() if device is None else int(device)
    layout = _abi.TqWorkspaceLayout()
    raise_for(lib.tq_mla_workspace_layout(ctypes.byref(params), dev, ctypes.byref(layout)))
    return layout


def _stream_handle(stream):
    if stream is None:
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


class MlaLaunch:
    """A validated dense paged MLA launch bound to its tensors and a workspace.

    The tensors are kept referenced for the lifetime of the object, so the numeric addresses in
    the validated params stay owned (docs/HOST-CONTRACTS.md:14-17).
    """

    def __init__(self, q, kv, page_table, seq_id, q_pos, kv_len, out, lse, *, scale,
                 query_counts, prefill=False, kv_format=None, workspace=None, idx=None,
                 k_len=None):
        self.tensors = (q, kv, page_table, seq_id, q_pos, kv_len, out, lse, idx, k_len)
        self.spec = make_spec(q, kv, page_table, seq_id, q_pos, kv_len, out, lse, scale=scale,
                              kv_format=kv_format)
        self.prefill = prefill
        if (idx is None) != (k_len is None):
            raise ValueError("a sparse plan needs both idx and k_len")
        if idx is not None and prefill:
            raise ValueError("sparse top-k plans are decode plans (no prefill form)")
        sparse = None if idx is None else (spec_of(idx), spec_of(k_len))
        self.params = validate(self.spec, query_counts, prefill=prefill,
                               idx=sparse[0] if sparse else None,
                               k_len=sparse[1] if sparse else None)
        self.out, self.lse = out, lse
        need = workspace_bytes(self.params, q.device.index) if self.params.should_launch else 0
        if workspace is None:
            workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=q.device)
        if workspace.numel() < need:
            raise TqError(102, "workspace")
        self.workspace = workspace

    def __call__(self, stream=None):
        err = _abi.TqContractError()
        fn = lib.tq_mla_prefill if self.prefill else lib.tq_mla_decode
        st = fn(ctypes.byref(self.params), ctypes.c_void_p(self.workspace.data_ptr()),
                self.workspace.numel(), _stream_handle(stream), ctypes.byref(err))
        raise_for(st, err)
        return self.out, self.lse

    def device_error(self, stream=None):
        flags = ctypes.c_int32()
        raise_for(lib.tq_mla_read_device_error(ctypes.c_void_p(self.workspace.data_ptr()),
                                               _stream_handle(stream), ctypes.byref(flags)))
        return flags.value


def set_kernel_timer(begin=None, end=None):
    """Record ``begin``/``end`` (``torch.cuda.Event``, already recorded once so that they exist)
    around the attention kernel of later launches from this thread; no arguments switches it off.
    """
    if (begin is None) != (end is None):
        raise ValueError("set_kernel_timer needs both events or neither")
    b = ctypes.c_void_p(begin.cuda_event) if begin is not None else None
    e = ctypes.c_void_p(end.cuda_event) if end is not None else None
    raise_for(lib.tq_mla_set_kernel_timer(b, e))


def mla_decode(q, kv, page_table, seq_id, q_pos, kv_len, *, scale, query_counts=None, out=None,
               lse=None, out_dtype=torch.bfloat16, prefill=False, kv_format=None, stream=None,
               idx=None, k_len=None):
    """Paged absorbed-MLA attention: returns ``(out [T,H,512], lse [T,H])``.

    Dense: token ``t`` attends to positions ``[0, min(kv_len[seq_id[t]], q_pos[t] + 1))`` of its
    sequence, whose rows live in ``kv`` pages listed by ``page_table[seq_id[t]]``. Sparse (``idx``
    i32 ``[T, K]`` and ``k_len`` i32 ``[T]`` given): token ``t`` attends to the positions
    ``idx[t, j]`` with ``j < k_len[t]``, ``0 <= idx <= q_pos[t]`` and ``idx < kv_len``.
    """
    t, h = q.shape[0], q.shape[1]
    if out is None:
        out = torch.empty((t, h, 512), dtype=out_dtype, device=q.device)
    if lse is None:
        lse = torch.empty((t, h), dtype=torch.float32, device=q.device)
    if query_counts is None:
        query_counts = torch.bincount(seq_id.cpu().long(), minlength=page_table.shape[0]).tolist()
    launch = MlaLaunch(q, kv, page_table, seq_id, q_pos, kv_len, out, lse, scale=scale,
                       query_counts=query_counts, prefill=prefill, kv_format=kv_format, idx=idx,
                       k_len=k_len)
    return launch(stream)


def kv_write_spec(src, kv, page_table, seq_id, pos, *, kv_format=None, norm_weight=None,
                  norm_eps=1e-6):
    """Declaration of a KV-writer call: ``src`` bf16 ``[T, W]`` rows into the paged pool ``kv``."""
    if kv_format is None:
        kv_format = _abi.KV_BF16_ROPE576 if src.shape[-1] == 576 else _abi.KV_BF16
    s = _abi.TqKvWriteSpec()
    s.src = spec_of(src)
    s.kv = pool_spec(kv, kv_format)
    s.page_table = spec_of(page_table)
    s.seq_id = spec_of(seq_id)
    s.pos = spec_of(pos)
    s.kv_format = kv_format
    if norm_weight is not None:
        s.norm_weight = spec_of(norm_weight)
        s.norm_eps = float(norm_eps)
    return s


def kv_write(src, kv, page_table, seq_id, pos, *, kv_format=None, flags=None, stream=None,
             norm_weight=None, norm_eps=1e-6):
    """Write row ``t`` of ``src`` to position ``pos[t]`` of sequence ``seq_id[t]`` in ``kv``.

    bf16 formats copy the row; ``KV_FP8_E4M3`` quantizes it per 128-value tile (codes plus f32
    scales). With ``norm_weight`` (bf16 ``[512]``) the row's 512 latent values are RMS-normalised
    first (``norm_eps`` > 0). ``flags`` is an optional device ``int32`` tensor that collects the
    range flags of skipped rows (``TQ_DEV_*``).
    """
    s = kv_write_spec(src, kv, page_table, seq_id, pos, kv_format=kv_format,
                      norm_weight=norm_weight, norm_eps=norm_eps)
    err = _abi.TqContractError()
    fp = ctypes.c_void_p(flags.data_ptr()) if flags is not None else None
    raise_for(lib.tq_kv_write(ctypes.byref(s), fp, _stream_handle(stream), ctypes.byref(err)), err)
    return kv


def prologue_spec(x, w_qa, q_norm, w_qb, w_uk, w_kva, kv_norm, pos, seq_id, page_table, kv, q, *,
                  heads, nope_dim, rope_dim, kv_format=None, q_eps=1e-6, kv_eps=1e-6,
                  rope_theta=10000.0):
    """Declaration of an MLA prologue call (``tq_mla_prologue``)."""
    if kv_format is None:
        kv_format = _abi.KV_BF16_ROPE576 if rope_dim else _abi.KV_BF16
    s = _abi.TqPrologueSpec()
    for name, t in (("x", x), ("w_qa", w_qa), ("q_norm", q_norm), ("w_qb", w_qb), ("w_uk", w_uk),
                    ("w_kva", w_kva), ("kv_norm", kv_norm), ("pos", pos), ("seq_id", seq_id),
                    ("page_table", page_table), ("q", q)):
        setattr(s, name, spec_of(t))
    s.kv = pool_spec(kv, kv_format)
    s.heads, s.nope_dim, s.rope_dim, s.kv_format = int(heads), int(nope_dim), int(rope_dim), kv_format
    s.q_eps, s.kv_eps, s.rope_theta = float(q_eps), float(kv_eps), float(rope_theta)
    return s


class MlaPrologue:
    """A validated prologue: token activations ``x`` to absorbed queries ``q`` and cache rows.

    ``x`` bf16 ``[T, Dm]``; weights ``w_qa [Rq, Dm]``, ``q_norm [Rq]``, ``w_qb [H (Dn + Dr), Rq]``,
    ``w_uk [H, Dn, 512]``, ``w_kva [512 + Dr, Dm]``, ``kv_norm [512]``; ``pos``/``seq_id`` i32
    ``[T]``. Writes ``q`` bf16 ``[T, H, 512 + Dr]`` and each token's row into the paged pool
    ``kv`` at ``pos`` of sequence ``seq_id`` (``kv_format`` rows). Owns only its workspace.
    """

    def __init__(self, x, w_qa, q_norm, w_qb, w_uk, w_kva, kv_norm, pos, seq_id, page_table, kv,
                 q, **kw):
        self._keep = (x, w_qa, q_norm, w_qb, w_uk, w_kva, kv_norm, pos, seq_id, page_table, kv, q)
        self.spec = prologue_spec(x, w_qa, q_norm, w_qb, w_uk, w_kva, kv_norm, pos, seq_id,
                                  page_table, kv, q, **kw)
        err = _abi.TqContractError()
        raise_for(lib.tq_mla_prologue_validate(ctypes.byref(self.spec), ctypes.byref(err)), err)
        nbytes = ctypes.c_uint64()
        raise_for(lib.tq_mla_prologue_workspace_bytes(ctypes.byref(self.spec),
                                                      ctypes.byref(nbytes)))
        self.workspace = torch.empty(int(nbytes.value), dtype=torch.uint8, device=x.device)
        self.q = q

    def __call__(self, flags=None, stream=None):
        err = _abi.TqContractError()
        fp = ctypes.c_void_p(flags.data_ptr()) if flags is not None else None
        raise_for(lib.tq_mla_prologue(ctypes.byref(self.spec),
                                      ctypes.c_void_p(self.workspace.data_ptr()),
                                      self.workspace.numel(), fp, _stream_handle(stream),
                                      ctypes.byref(err)), err)
        return self.q


def mla_prologue(x, w_qa, q_norm, w_qb, w_uk, w_kva, kv_norm, pos, seq_id, page_table, kv, *,
                 heads, nope_dim, rope_dim, q=None, flags=None, stream=None, **kw):
    """One prologue call (see ``MlaPrologue``); returns ``q``."""
    if q is None:
        q = torch.empty((x.shape[0], heads, 512 + rope_dim), dtype=torch.bfloat16, device=x.device)
    return MlaPrologue(x, w_qa, q_norm, w_qb, w_uk, w_kva, kv_norm, pos, seq_id, page_table, kv, q,
                       heads=heads, nope_dim=nope_dim, rope_dim=rope_dim, **kw)(flags, stream)


def combine_parts(part_out, part_lse, out=None, lse=None, stream=None):
    """Merge ``G`` partial results (``part_out f32 [G,T,H,512]``, ``part_lse f32 [G,T,H]``)."""
    g, t, h, _ = part_out.shape
    if out is None:
        out = torch.empty((t, h, 512), dtype=torch.bfloat16, device=part_out.device)
    if lse is None:
        lse = torch.empty((t, h), dtype=torch.float32, device=part_out.device)
    p = _abi.TqCombineParams()
    p.parts, p.tokens, p.heads = g, t, h
    p.part_out, p.part_lse = part_out.data_ptr(), part_lse.data_ptr()
    p.out, p.lse = out.data_ptr(), lse.data_ptr()
    p.out_stride_token = out.stride(0) * out.element_size()
    p.out_stride_head = out.stride(1) * out.element_size()
    p.out_dtype = _TORCH_DTYPE[out.dtype]
    raise_for(lib.tq_mla_combine(ctypes.byref(p), _stream_handle(stream)))
    return out, lse


def default_scale(width):
    """1/sqrt(192) for 576-wide rows (DeepSeek-style 128 + 64 query-key width); 0.0625 for 512."""
    return 1.0 / math.sqrt(192.0) if width == 576 else 0.0625
