"""Host validation of the KV writer (tq_kv_write_validate), CPU only: fake numeric addresses,
the same field names and violation kinds as the attention contract."""

import ctypes

import pytest

from tq_mla import _abi

SHAPE, DTYPE, STRIDE, ALIGNMENT, ADDRESS, CAPACITY, ALIAS = 1, 2, 4, 5, 6, 7, 12
GiB = 1 << 30


def tensor(shape, strides, dtype, address, capacity=None):
    t = _abi.TqTensorSpec()
    t.rank = len(shape)
    for i, (d, s) in enumerate(zip(shape, strides)):
        t.shape[i], t.strides_bytes[i] = d, s
    t.dtype = dtype
    t.device_address = address
    if capacity is None:
        capacity = sum((d - 1) * s for d, s in zip(shape, strides)) + (strides[-1] if shape else 0)
    t.buffer_bytes = capacity
    return t


def spec(rows=5, fmt=_abi.KV_FP8_E4M3, width=None, src_stride=None, src_addr=1 * GiB,
         row=544, pages=7, seqs=3, slots=4):
    width = width or (576 if fmt == _abi.KV_BF16_ROPE576 else 512)
    payload = {0: 1024, 1: 528, 2: 1152}[fmt]
    s = _abi.TqKvWriteSpec()
    s.src = tensor([rows, width], [src_stride or 2 * width, 2], _abi.DTYPE_BF16, src_addr)
    s.kv = tensor([pages, 64, payload], [64 * row, row, 1], _abi.DTYPE_U8, 2 * GiB,
                  pages * 64 * row)
    s.page_table = tensor([seqs, slots], [4 * slots, 4], _abi.DTYPE_I32, 3 * GiB)
    s.seq_id = tensor([rows], [4], _abi.DTYPE_I32, 4 * GiB)
    s.pos = tensor([rows], [4], _abi.DTYPE_I32, 5 * GiB)
    s.kv_format = fmt
    return s


def verdict(s):
    err = _abi.TqContractError()
    st = _abi.lib.tq_kv_write_validate(ctypes.byref(s), ctypes.byref(err))
    return None if st == 0 else (err.field.decode(), st)


@pytest.mark.parametrize("fmt,row", [(_abi.KV_FP8_E4M3, 528), (_abi.KV_FP8_E4M3, 544),
                                     (_abi.KV_BF16, 1024), (_abi.KV_BF16_ROPE576, 1152),
                                     (_abi.KV_BF16_ROPE576, 1168)])
def test_supported_formats_and_strides(fmt, row):
    assert verdict(spec(fmt=fmt, row=row)) is None


def test_rejections_name_the_field_and_kind():
    s = spec(); s.kv_format = 7
    assert verdict(s) == ("kv_format", SHAPE)
    assert verdict(spec(width=576)) == ("src", SHAPE)           # FP8 rows take 512 values
    s = spec(); s.src.dtype = _abi.DTYPE_F32
    assert verdict(s) == ("src", DTYPE)
    assert verdict(spec(src_stride=1032)) == ("src", STRIDE)    # not a multiple of 16
    assert verdict(spec(src_stride=1000)) == ("src", STRIDE)    # shorter than a row
    assert verdict(spec(src_addr=GiB + 8)) == ("src", ALIGNMENT)
    assert verdict(spec(row=536)) == ("kv", STRIDE)             # row stride % 16
    assert verdict(spec(row=512)) == ("kv", STRIDE)             # shorter than the payload
    s = spec(); s.pos.shape[0] = 4
    assert verdict(s) == ("pos", SHAPE)
    s = spec(); s.seq_id.dtype = _abi.DTYPE_U8
    assert verdict(s) == ("seq_id", DTYPE)
    s = spec(); s.page_table.strides_bytes[0] = 20
    assert verdict(s) == ("page_table", STRIDE)
    s = spec()  # the pool must reach the last row's last payload byte, not its padding
    s.kv.buffer_bytes = 6 * 64 * 544 + 63 * 544 + 528
    assert verdict(s) is None
    s.kv.buffer_bytes -= 1
    assert verdict(s) == ("kv", CAPACITY)
    s = spec(); s.pos.device_address = 0
    assert verdict(s) == ("pos", ADDRESS)


def test_inputs_may_not_overlap_the_pool():
    s = spec()
    s.src.device_address = s.kv.device_address + 64 * 544  # inside page 1
    assert verdict(s) == ("kv", ALIAS)  # the overlapping output is named, as in the reference


def test_empty_call_needs_no_storage():
    s = spec(rows=0)
    for name in ("src", "seq_id", "pos"):
        getattr(s, name).device_address = 0
        getattr(s, name).buffer_bytes = 0
    assert verdict(s) is None
    err = _abi.TqContractError()
    assert _abi.lib.tq_kv_write(ctypes.byref(s), None, None, ctypes.byref(err)) == 0


def test_norm_weight_and_eps():
    s = spec()
    s.norm_weight = tensor([512], [2], _abi.DTYPE_BF16, 6 * GiB)
    s.norm_eps = 1e-6
    assert verdict(s) is None
    s.norm_eps = 0.0
    assert verdict(s) == ("norm_eps", 10)
    s.norm_eps = float("nan")
    assert verdict(s) == ("norm_eps", 10)
    s = spec()
    s.norm_weight = tensor([576], [2], _abi.DTYPE_BF16, 6 * GiB)
    s.norm_eps = 1e-6
    assert verdict(s) == ("norm_weight", SHAPE)
    s = spec()
    s.norm_weight = tensor([512], [2], _abi.DTYPE_BF16, 6 * GiB + 8)
    s.norm_eps = 1e-6
    assert verdict(s) == ("norm_weight", ALIGNMENT)
    s = spec()
    s.norm_weight = tensor([512], [2], _abi.DTYPE_BF16, 2 * GiB + 4096)  # inside the pool
    s.norm_eps = 1e-6
    assert verdict(s) == ("kv", ALIAS)
