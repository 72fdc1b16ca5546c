"""ctypes binding of ``include/tq_mla.h`` (libtq_mla.so, built in-tree by ``tq_mla.build``).

Importing this module loads the native library and fails loudly when it is missing: there is no
Python or CPU fallback for any launch.
"""

import ctypes
import os
from pathlib import Path

LIB_NAME = "libtq_mla.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

DTYPE_BF16, DTYPE_I32, DTYPE_F32, DTYPE_U8 = 0, 1, 2, 3
KV_BF16, KV_FP8_E4M3, KV_BF16_ROPE576 = 0, 1, 2

STATUS = {
    0: "ok", 1: "Shape", 2: "Dtype", 3: "Dimension", 4: "Stride", 5: "Alignment", 6: "Address",
    7: "Capacity", 8: "Overflow", 9: "QueryCount", 10: "Scale", 11: "Group", 12: "Alias",
    100: "InvalidArgument", 101: "Unsupported", 102: "Workspace", 103: "Cuda", 104: "Params",
    105: "Range", 106: "Comm",
}
DEV_WAIT_TIMEOUT, DEV_PAGE_RANGE, DEV_SEQ_RANGE, DEV_TABLE_SHORT, DEV_WORK_OVERFLOW = 1, 2, 4, 8, 16


class TqTensorSpec(ctypes.Structure):
    _fields_ = [
        ("shape", ctypes.c_uint64 * 3),
        ("strides_bytes", ctypes.c_uint64 * 3),
        ("rank", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("device_address", ctypes.c_uint64),
        ("buffer_bytes", ctypes.c_uint64),
    ]


SPEC_FIELDS = ("q", "kv", "page_table", "seq_id", "q_pos", "kv_len", "out", "lse")


class TqMlaSpec(ctypes.Structure):
    _fields_ = [(name, TqTensorSpec) for name in SPEC_FIELDS] + [
        ("kv_format", ctypes.c_int32),
        ("softmax_scale", ctypes.c_float),
    ]


class TqContractError(ctypes.Structure):
    _fields_ = [("field", ctypes.c_char_p), ("kind", ctypes.c_int32)]


class TqMlaParams(ctypes.Structure):
    _fields_ = [
        ("spec", TqMlaSpec),
        ("tokens", ctypes.c_uint64), ("heads", ctypes.c_uint64), ("sequences", ctypes.c_uint64),
        ("slots", ctypes.c_uint64), ("pages", ctypes.c_uint64), ("qk_width", ctypes.c_uint64),
        ("row_stride", ctypes.c_uint64),
        ("max_queries_per_sequence", ctypes.c_int32),
        ("should_launch", ctypes.c_int32),
        ("idx", TqTensorSpec), ("k_len", TqTensorSpec),
        ("topk", ctypes.c_uint64), ("sparse", ctypes.c_int32), ("reserved", ctypes.c_int32),
        ("digest", ctypes.c_uint64),
    ]


class TqCombineParams(ctypes.Structure):
    _fields_ = [
        ("parts", ctypes.c_uint64), ("tokens", ctypes.c_uint64), ("heads", ctypes.c_uint64),
        ("part_out", ctypes.c_uint64), ("part_lse", ctypes.c_uint64),
        ("out", ctypes.c_uint64), ("lse", ctypes.c_uint64),
        ("out_stride_token", ctypes.c_uint64), ("out_stride_head", ctypes.c_uint64),
        ("out_dtype", ctypes.c_int32),
    ]


class TqCommId(ctypes.Structure):
    _fields_ = [("internal", ctypes.c_char * 128)]


class TqContextMergeParams(ctypes.Structure):
    _fields_ = [(name, ctypes.c_uint64) for name in (
        "tokens", "heads", "part_out", "part_lse", "gather_out", "gather_lse", "gather_out_bytes",
        "gather_lse_bytes", "out", "lse", "out_stride_token", "out_stride_head")] + [
        ("out_dtype", ctypes.c_int32)]


class TqWorkspaceLayout(ctypes.Structure):
    _fields_ = [(name, ctypes.c_uint64) for name in (
        "total_bytes", "header", "unit_n", "unit_pages", "unit_gstart", "unit_first",
        "unit_nsplit", "unit_split_off", "pair_begin", "combine_list", "empty_list", "part_lse",
        "part_out", "sparse_rows", "sparse_count")] + [("pairs", ctypes.c_int32)]


class TqKvWriteSpec(ctypes.Structure):
    _fields_ = [(name, TqTensorSpec) for name in ("src", "kv", "page_table", "seq_id", "pos")] + [
        ("kv_format", ctypes.c_int32), ("norm_weight", TqTensorSpec), ("norm_eps", ctypes.c_float)]


class TqPrologueSpec(ctypes.Structure):
    _fields_ = [(name, TqTensorSpec) for name in (
        "x", "w_qa", "q_norm", "w_qb", "w_uk", "w_kva", "kv_norm", "pos", "seq_id", "page_table",
        "kv", "q")] + [(name, ctypes.c_int32) for name in (
            "heads", "nope_dim", "rope_dim", "kv_format")] + [(name, ctypes.c_float) for name in (
                "q_eps", "kv_eps", "rope_theta")]


# Every exported symbol of include/tq_mla.h, with its ctypes prototype.
_P = ctypes.POINTER
_U64, _I32, _VP = ctypes.c_uint64, ctypes.c_int32, ctypes.c_void_p
PROTOTYPES = {
    "tq_mla_validate": (_I32, [_P(TqMlaSpec), _P(ctypes.c_uint8), _U64, _P(TqMlaParams),
                               _P(TqContractError)]),
    "tq_mla_prefill_validate": (_I32, [_P(TqMlaSpec), _P(ctypes.c_uint32), _U64,
                                       _P(TqMlaParams), _P(TqContractError)]),
    "tq_mla_should_launch": (_I32, [_P(TqMlaParams)]),
    "tq_mla_sparse_validate": (_I32, [_P(TqMlaSpec), _P(TqTensorSpec), _P(TqTensorSpec),
                                      _P(ctypes.c_uint8), _U64, _P(TqMlaParams),
                                      _P(TqContractError)]),
    "tq_mla_workspace_bytes": (_I32, [_P(TqMlaParams), _I32, _P(_U64)]),
    "tq_mla_workspace_layout": (_I32, [_P(TqMlaParams), _I32, _P(TqWorkspaceLayout)]),
    "tq_mla_decode": (_I32, [_P(TqMlaParams), _VP, _U64, _VP, _P(TqContractError)]),
    "tq_mla_prefill": (_I32, [_P(TqMlaParams), _VP, _U64, _VP, _P(TqContractError)]),
    "tq_mla_combine": (_I32, [_P(TqCombineParams), _VP]),
    "tq_mla_read_device_error": (_I32, [_VP, _VP, _P(_I32)]),
    "tq_comm_unique_id": (_I32, [_P(TqCommId)]),
    "tq_comm_init": (_I32, [_P(TqCommId), _I32, _I32, _P(_VP)]),
    "tq_comm_abort": (_I32, [_VP]),
    "tq_comm_destroy": (_I32, [_VP]),
    "tq_comm_rank": (_I32, [_VP, _P(_I32), _P(_I32)]),
    "tq_mla_context_merge": (_I32, [_P(TqContextMergeParams), _VP, _VP]),
    "tq_peer_merge_create": (_I32, [_VP, _U64, _U64, _P(_VP)]),
    "tq_peer_merge_partials": (_I32, [_VP, _P(_U64), _P(_U64)]),
    "tq_peer_merge": (_I32, [_VP, _U64, _U64, _U64, _U64, _I32, _VP]),
    "tq_peer_merge_read_error": (_I32, [_VP, _VP, _P(_I32)]),
    "tq_peer_merge_destroy": (_I32, [_VP]),
    "tq_mla_set_kernel_timer": (_I32, [_VP, _VP]),
    "tq_mla_decode_no_alloc": (_I32, [_P(TqMlaParams), _VP, _P(TqContractError)]),
    "tq_mla_no_alloc_read_device_error": (_I32, [_VP, _P(_I32)]),
    "tq_kv_write_validate": (_I32, [_P(TqKvWriteSpec), _P(TqContractError)]),
    "tq_kv_write": (_I32, [_P(TqKvWriteSpec), _VP, _VP, _P(TqContractError)]),
    "tq_mla_prologue_validate": (_I32, [_P(TqPrologueSpec), _P(TqContractError)]),
    "tq_mla_prologue_workspace_bytes": (_I32, [_P(TqPrologueSpec), _P(_U64)]),
    "tq_mla_prologue": (_I32, [_P(TqPrologueSpec), _VP, _U64, _VP, _VP, _P(TqContractError)]),
    "tq_philox_block": (None, [_P(ctypes.c_uint32), _P(ctypes.c_uint32), _P(ctypes.c_uint32)]),
    "tq_philox_words": (_I32, [_U64, _U64, _U64, _P(ctypes.c_uint32), _U64]),
    "tq_philox_uniform_f32": (ctypes.c_float, [ctypes.c_uint32]),
    "tq_gen_normal_bf16": (_I32, [_VP, _U64, _U64, _U64, _U64, _VP]),
    "tq_gen_kv_pool": (_I32, [_VP, _U64, _U64, _U64, _VP, _U64, _VP, _VP, _U64, _U64, _VP]),
    "tq_mla_status_string": (ctypes.c_char_p, [_I32]),
    "tq_mla_version": (ctypes.c_char_p, []),
}


def _load():
    path = Path(os.environ.get("TQ_MLA_LIB", LIB_PATH))
    if not path.exists():
        raise ImportError(
            f"{path} is missing: build it with `python -m tq_mla.build` (nvcc, sm_100a). "
            "There is no fallback implementation."
        )
    lib = ctypes.CDLL(str(path))
    for name, (res, args) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


class TqError(RuntimeError):
    """A non-contract failure reported by the library (CUDA, workspace, params)."""

    def __init__(self, status, field=None):
        self.status = status
        self.field = field
        name = STATUS.get(status, str(status))
        super().__init__(f"{field}: {name}" if field else name)


class ContractError(ValueError):
    """A rejected contract: ``field`` and ``kind`` mirror ``ContractError`` in tq-core."""

    def __init__(self, field, kind):
        self.field = field
        self.kind = kind
        super().__init__(f"{field}: {STATUS.get(kind, kind)}")


def raise_for(status, err=None):
    if status == 0:
        return
    field = err.field.decode() if err is not None and err.field else None
    if 1 <= status <= 12:
        raise ContractError(field, status)
    raise TqError(status, field)
