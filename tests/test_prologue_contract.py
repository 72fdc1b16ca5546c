"""Host validation of the MLA prologue (tq_mla_prologue_validate, tq_mla_prologue_workspace_bytes),
CPU only: fake numeric addresses, the field names and violation kinds of the other contracts."""

import ctypes

import pytest

from tq_mla import _abi

SHAPE, DTYPE, ALIGNMENT, SCALE, ALIAS = 1, 2, 5, 10, 12
GiB = 1 << 30


def tensor(shape, dtype, address, elem):
    t = _abi.TqTensorSpec()
    t.rank = len(shape)
    stride = elem
    strides = []
    for d in reversed(shape):
        strides.append(stride)
        stride *= d
    for i, (d, s) in enumerate(zip(shape, reversed(strides))):
        t.shape[i], t.strides_bytes[i] = d, s
    t.dtype = dtype
    t.device_address = address
    t.buffer_bytes = stride
    return t


def spec(tokens=6, dm=256, rq=64, heads=4, dn=128, dr=64, fmt=None, pages=5, seqs=2, slots=3):
    fmt = (_abi.KV_BF16_ROPE576 if dr else _abi.KV_BF16) if fmt is None else fmt
    width = 512 + dr
    bf, i32 = _abi.DTYPE_BF16, _abi.DTYPE_I32
    s = _abi.TqPrologueSpec()
    s.x = tensor([tokens, dm], bf, 1 * GiB, 2)
    s.w_qa = tensor([rq, dm], bf, 2 * GiB, 2)
    s.q_norm = tensor([rq], bf, 3 * GiB, 2)
    s.w_qb = tensor([heads * (dn + dr), rq], bf, 4 * GiB, 2)
    s.w_uk = tensor([heads, dn, 512], bf, 5 * GiB, 2)
    s.w_kva = tensor([width, dm], bf, 6 * GiB, 2)
    s.kv_norm = tensor([512], bf, 7 * GiB, 2)
    s.pos = tensor([tokens], i32, 8 * GiB, 4)
    s.seq_id = tensor([tokens], i32, 9 * GiB, 4)
    s.page_table = tensor([seqs, slots], i32, 10 * GiB, 4)
    payload = {0: 1024, 1: 528, 2: 1152}[fmt]
    row = (payload + 15) // 16 * 16
    kv = _abi.TqTensorSpec()
    kv.rank = 3
    for i, (d, st) in enumerate(zip([pages, 64, payload], [64 * row, row, 1])):
        kv.shape[i], kv.strides_bytes[i] = d, st
    kv.dtype = _abi.DTYPE_U8
    kv.device_address = 11 * GiB
    kv.buffer_bytes = pages * 64 * row
    s.kv = kv
    s.q = tensor([tokens, heads, width], bf, 12 * GiB, 2)
    s.heads, s.nope_dim, s.rope_dim, s.kv_format = heads, dn, dr, fmt
    s.q_eps, s.kv_eps, s.rope_theta = 1e-6, 1e-6, 10000.0
    return s


def verdict(s):
    err = _abi.TqContractError()
    st = _abi.lib.tq_mla_prologue_validate(ctypes.byref(s), ctypes.byref(err))
    return None if st == 0 else (err.field.decode(), st)


@pytest.mark.parametrize("dr,fmt", [(0, _abi.KV_BF16), (0, _abi.KV_FP8_E4M3),
                                    (64, _abi.KV_BF16_ROPE576)])
def test_both_row_forms_validate(dr, fmt):
    assert verdict(spec(dr=dr, fmt=fmt)) is None
    # the model sizes: no-RoPE 64 x 256 over hidden 4096, RoPE 128 x 128 over hidden 7168
    assert verdict(spec(dm=4096, rq=1536, heads=64, dn=256, dr=0, fmt=fmt if not dr else 0)) is None
    assert verdict(spec(dm=7168, rq=1536, heads=128, dn=128, dr=64)) is None


def test_rejections_name_the_field_and_kind():
    assert verdict(spec(dr=32)) == ("rope_dim", SHAPE)
    assert verdict(spec(dr=0, fmt=_abi.KV_BF16_ROPE576)) == ("kv_format", SHAPE)
    assert verdict(spec(dr=64, fmt=_abi.KV_FP8_E4M3)) == ("kv_format", SHAPE)
    s = spec(); s.kv_format = 9
    assert verdict(s) == ("kv_format", SHAPE)
    s = spec(); s.heads = 0
    assert verdict(s) == ("heads", SHAPE)
    s = spec(); s.heads = 129
    assert verdict(s) == ("heads", SHAPE)
    assert verdict(spec(dn=12)) == ("nope_dim", SHAPE)
    assert verdict(spec(dm=100)) == ("x", SHAPE)
    assert verdict(spec(rq=20)) == ("w_qa", SHAPE)
    s = spec(); s.w_qb.shape[0] -= 1
    assert verdict(s) == ("w_qb", SHAPE)
    s = spec(); s.w_uk.shape[2] = 576
    assert verdict(s) == ("w_uk", SHAPE)
    s = spec(); s.q.shape[2] = 512
    assert verdict(s) == ("q", SHAPE)
    s = spec(); s.kv_norm.dtype = _abi.DTYPE_F32
    assert verdict(s) == ("kv_norm", DTYPE)
    s = spec(); s.pos.dtype = _abi.DTYPE_BF16
    assert verdict(s) == ("pos", DTYPE)
    s = spec(); s.x.device_address += 8
    assert verdict(s) == ("x", ALIGNMENT)
    s = spec(); s.q_eps = 0.0
    assert verdict(s) == ("q_eps", SCALE)
    s = spec(); s.kv_eps = float("nan")
    assert verdict(s) == ("kv_eps", SCALE)
    s = spec(); s.rope_theta = 1.0
    assert verdict(s) == ("rope_theta", SCALE)


def test_output_aliasing_an_input_is_rejected():
    s = spec(); s.q.device_address = s.x.device_address
    assert verdict(s)[1] == ALIAS
    s = spec(); s.kv.device_address = s.w_qa.device_address
    assert verdict(s)[1] == ALIAS


def test_empty_batch_validates_with_unset_addresses():
    s = spec(tokens=0)
    for name in ("x", "pos", "seq_id", "q"):
        getattr(s, name).device_address = 0
    assert verdict(s) is None


def test_workspace_holds_the_intermediates_and_blas_scratch():
    n = ctypes.c_uint64()
    s = spec(tokens=6, rq=64, heads=4, dn=128, dr=64)
    assert _abi.lib.tq_mla_prologue_workspace_bytes(ctypes.byref(s), ctypes.byref(n)) == 0
    r = lambda v: (v + 255) // 256 * 256
    want = r(6 * 64 * 2) + r(6 * 4 * 192 * 2) + r(6 * 576 * 2) + (32 << 20)
    assert n.value == want
    bad = spec(dr=32)
    assert _abi.lib.tq_mla_prologue_workspace_bytes(ctypes.byref(bad), ctypes.byref(n)) == SHAPE
