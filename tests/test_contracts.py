"""Host contract: the C++ validator (tq_mla_validate) against the oracle restatement.

Cases mirror crates/tq-core/tests/host_acceptance.rs (the reference's independent acceptance of
SmlaParams::new) on fake numeric addresses (slot << 48, tests/support/mod.rs:30-46), plus the
documented generalisations (576-wide rows, 16/128 heads, runtime scale for the 576 format,
prefill plans, f32 partial outputs). Every case asserts that both implementations give the same
verdict and that the verdict is the expected one.
"""

import ctypes
import math
import struct

import numpy as np
import pytest

from oracle import contracts as oc
from oracle import philox as op
from tq_mla import _abi

FIELDS = oc.FIELDS
U64 = (1 << 64) - 1


def to_c(spec: oc.Spec):
    c = _abi.TqMlaSpec()
    for name in FIELDS:
        t = getattr(spec, name)
        ct = getattr(c, name)
        ct.rank = len(t.shape)
        for i in range(3):
            ct.shape[i] = int(t.shape[i]) & U64 if i < len(t.shape) else 0
            ct.strides_bytes[i] = int(t.strides[i]) & U64 if i < len(t.strides) else 0
        ct.dtype = t.dtype
        ct.device_address = int(t.address) & U64
        ct.buffer_bytes = int(t.capacity) & U64
    c.kv_format = spec.kv_format
    c.softmax_scale = spec.scale
    return c


def c_verdict(spec, counts, prefill=False):
    c = to_c(spec)
    err = _abi.TqContractError()
    params = _abi.TqMlaParams()
    if prefill:
        arr = (ctypes.c_uint32 * max(1, len(counts)))(*counts)
        st = _abi.lib.tq_mla_prefill_validate(ctypes.byref(c), arr, len(counts),
                                              ctypes.byref(params), ctypes.byref(err))
    else:
        arr = (ctypes.c_uint8 * max(1, len(counts)))(*[x & 0xFF for x in counts])
        st = _abi.lib.tq_mla_validate(ctypes.byref(c), arr, len(counts), ctypes.byref(params),
                                      ctypes.byref(err))
    if st == 0:
        return None, params
    return (err.field.decode(), st), params


def o_verdict(spec, counts, prefill=False):
    try:
        oc.validate(spec, counts, max_per_seq=None if prefill else oc.MAX_DECODE_QUERIES)
        return None
    except oc.ContractError as e:
        return (e.field, e.kind)


def check(spec, counts, expected=None, *, prefill=False):
    """Both verdicts agree; ``expected`` is ``None`` (accepted), ``(field, kind)`` or ``'reject'``."""
    cv, _ = c_verdict(spec, counts, prefill)
    ov = o_verdict(spec, counts, prefill)
    assert cv == ov, (cv, ov)
    if expected == "reject":
        assert cv is not None
    else:
        assert cv == expected, (cv, expected)


def smla(tokens, heads, sequences, fmt=oc.KV_BF16, **kw):
    return oc.make_spec(tokens, heads, sequences, kv_format=fmt, **kw)


def size_to_span(t):
    t.capacity = oc.wide_span(t)


def wrong_dtype(d):
    return oc.BF16 if d == oc.U8 else oc.U8


# ----------------------------------------------------------------------------- acceptance

@pytest.mark.parametrize("fmt,stride", [(oc.KV_BF16, 1024), (oc.KV_BF16, 1040),
                                        (oc.KV_BF16_ROPE576, 1152), (oc.KV_BF16_ROPE576, 1168),
                                        (oc.KV_FP8_E4M3, 528), (oc.KV_FP8_E4M3, 544),
                                        (oc.KV_FP8_E4M3, 560)])
@pytest.mark.parametrize("heads", [16, 32, 64, 128])
def test_supported_shapes_formats_and_capacity(fmt, stride, heads):
    for counts in ([1], [0, 1, 2, 3, 4], [4] * 16, [4] * 64):
        s = smla(sum(counts), heads, len(counts), fmt)
        s.kv.strides = [64 * stride, stride, 1]
        size_to_span(s.kv)
        check(s, counts, None)
        _, params = c_verdict(s, counts)
        assert params.should_launch == 1
        assert _abi.lib.tq_mla_should_launch(ctypes.byref(params)) == 1


def test_fixed_geometry_rejections():
    for heads in (0, 1, 31, 33, 48, 63, 65, 127, 256):
        check(smla(1, heads, 1), [1], ("q", oc.SHAPE))
    for dim in (0, 256, 511, 513, 576, 1024):
        s = smla(1, 32, 1)
        s.q.shape[2] = dim
        check(s, [1], ("q", oc.SHAPE))
    for dim in (512, 575, 577):
        s = smla(1, 32, 1, oc.KV_BF16_ROPE576)
        s.q.shape[2] = dim
        check(s, [1], ("q", oc.SHAPE))
    s = smla(1, 32, 1)
    s.kv.shape[1] = 65
    check(s, [1], ("kv", oc.SHAPE))
    for payload in (512, 528, 544, 1023, 1025, 1152):
        s = smla(1, 32, 1)
        s.kv.shape[2] = payload
        check(s, [1], ("kv", oc.SHAPE))
    s = smla(1, 32, 1)
    s.kv_format = oc.KV_FP8_E4M3
    check(s, [1], ("kv", oc.SHAPE))
    s = smla(1, 32, 1)
    s.kv_format = 7
    check(s, [1], ("kv_format", oc.SHAPE))


def _f32(bits):
    return struct.unpack("<f", struct.pack("<I", bits))[0]


def test_glm_formats_require_the_exact_scale_constant():
    glm = struct.unpack("<I", struct.pack("<f", 0.0625))[0]
    for scale in (0.0, -0.0, -0.0625, 1.0, 512 ** -0.5, math.nan, math.inf, -math.inf,
                  _f32(glm - 1), _f32(glm + 1)):
        for fmt in (oc.KV_BF16, oc.KV_FP8_E4M3):
            s = smla(1, 32, 1, fmt)
            if fmt == oc.KV_FP8_E4M3:
                s.kv.shape[2] = 528
                s.kv.strides = [64 * 528, 528, 1]
                size_to_span(s.kv)
            s.scale = scale
            check(s, [1], ("softmax_scale", oc.SCALE))


def test_rope_format_scale_is_any_finite_positive_f32():
    for scale in (192 ** -0.5, 0.0625, 1.0, 1e-30, 3.0e38):
        s = smla(1, 128, 1, oc.KV_BF16_ROPE576, scale=scale)
        check(s, [1], None)
    for scale in (0.0, -0.0, -1.0, math.nan, math.inf, -math.inf, 1e39):
        s = smla(1, 128, 1, oc.KV_BF16_ROPE576, scale=scale)
        check(s, [1], ("softmax_scale", oc.SCALE))


def test_host_query_plan_checks_each_sequence_and_total():
    for counts in ([], [4], [1, 1, 2], [0, 3], [1, 4], [5, 0], [255, 0]):
        check(smla(4, 32, 2), counts, ("query_counts", oc.QUERY_COUNT))
    check(smla(6, 32, 2), [3, 3], None)
    check(smla(6, 32, 2), [5, 1], ("query_counts", oc.QUERY_COUNT))
    check(smla(1, 32, 0), [], "reject")


def test_prefill_plans_lift_the_per_sequence_limit():
    s = smla(4096, 128, 2, oc.KV_BF16_ROPE576)
    check(s, [2048, 2048], None, prefill=True)
    check(s, [4096, 0], None, prefill=True)
    check(s, [2048, 2047], ("query_counts", oc.QUERY_COUNT), prefill=True)
    check(s, [2048], ("query_counts", oc.QUERY_COUNT), prefill=True)


@pytest.mark.parametrize("field", FIELDS)
def test_each_tensor_field(field):
    original = smla(4, 32, 2)
    counts = [2, 2]

    def fresh():
        return original.copy()

    s = fresh()
    getattr(s, field).dtype = wrong_dtype(getattr(s, field).dtype)
    check(s, counts, (field, oc.DTYPE))
    s = fresh()
    t = getattr(s, field)
    t.strides[-1] = 0
    check(s, counts, (field, oc.STRIDE))
    s = fresh()
    t = getattr(s, field)
    t.strides[-1] = 2 * oc.ELEMENT[t.dtype]
    check(s, counts, (field, oc.STRIDE))
    s = fresh()
    getattr(s, field).address = 0
    check(s, counts, (field, oc.ADDRESS))
    s = fresh()
    getattr(s, field).capacity -= 1
    check(s, counts, (field, oc.CAPACITY))
    s = fresh()
    getattr(s, field).capacity = U64
    check(s, counts, (field, oc.OVERFLOW))
    s = fresh()
    t = getattr(s, field)
    t.address += 1
    if oc.ELEMENT[t.dtype] > 1 or field == "kv":
        check(s, counts, (field, oc.ALIGNMENT))
    else:
        check(s, counts, None)
    s = fresh()
    getattr(s, field).shape[0] = 1 << 31
    check(s, counts, "reject")
    for axis in range(len(original.__dict__[field].shape)):
        s = fresh()
        getattr(s, field).shape[axis] = U64
        check(s, counts, "reject")


def test_dependent_shapes_are_not_inferred_away():
    for field, axis in (("seq_id", 0), ("q_pos", 0), ("kv_len", 0), ("out", 0), ("out", 1),
                        ("out", 2), ("lse", 0), ("lse", 1)):
        s = smla(4, 32, 2)
        getattr(s, field).shape[axis] += 1
        check(s, [2, 2], (field, oc.SHAPE))


def test_kv_row_stride_and_exact_last_byte():
    for fmt, payload, strides in ((oc.KV_BF16, 1024, (1024, 1040, 2048)),
                                  (oc.KV_BF16_ROPE576, 1152, (1152, 1168, 1280)),
                                  (oc.KV_FP8_E4M3, 528, (528, 544, 560, 1024))):
        for stride in strides:
            s = smla(1, 32, 1, fmt)
            s.kv.shape[2] = payload
            s.kv.strides = [64 * stride, stride, 1]
            size_to_span(s.kv)
            assert s.kv.capacity == (17 * 64 - 1) * stride + payload
            check(s, [1], None)
            s.kv.capacity -= 1
            check(s, [1], ("kv", oc.CAPACITY))
    for stride in (0, 16, 512, 527, 529, 543, 545):
        s = smla(1, 32, 1, oc.KV_FP8_E4M3)
        s.kv.shape[2] = 528
        s.kv.strides = [64 * stride, stride, 1]
        size_to_span(s.kv)
        check(s, [1], ("kv", oc.STRIDE))
    s = smla(1, 32, 1)
    s.kv.strides[0] += 16
    check(s, [1], ("kv", oc.STRIDE))
    s = smla(1, 32, 1)
    s.kv.strides[1] = 1008
    check(s, [1], ("kv", oc.STRIDE))
    s = smla(1, 32, 1, oc.KV_BF16_ROPE576)
    s.kv.strides = [64 * 1160, 1160, 1]
    check(s, [1], ("kv", oc.STRIDE))


def test_padded_q_and_out_with_natural_alignment():
    s = smla(4, 32, 2)
    for t, inner in ((s.q, 1030), (s.out, 1030)):
        t.strides = [32 * inner + 6, inner, 2]
        t.address += 2
        size_to_span(t)
    s.kv.address += 16
    check(s, [2, 2], None)
    good = s.copy()
    s.q.strides[0] = 32 * 1030 - 2
    check(s, [2, 2], ("q", oc.STRIDE))
    s = good.copy()
    s.q.strides[1] = 1023
    check(s, [2, 2], ("q", oc.STRIDE))
    s = good.copy()
    s.out.strides[1] = 1031
    check(s, [2, 2], ("out", oc.STRIDE))
    s = good.copy()
    s.lse.strides[0] += 4
    check(s, [2, 2], ("lse", oc.STRIDE))
    s = good.copy()
    s.page_table.strides[0] += 4
    check(s, [2, 2], ("page_table", oc.STRIDE))


def test_empty_launch_skips_storage_but_keeps_metadata_checks():
    s = smla(0, 32, 0)
    for f in FIELDS:
        getattr(s, f).address = 0
        getattr(s, f).capacity = 0
    check(s, [], None)
    _, params = c_verdict(s, [])
    assert params.should_launch == 0
    s.q.shape[2] = 513
    check(s, [], ("q", oc.SHAPE))
    check(smla(0, 32, 1), [1], ("query_counts", oc.QUERY_COUNT))


def test_empty_cache_inside_nonempty_batch():
    s = smla(1, 32, 1)
    s.kv = oc.packed_tensor([0, 64, 1024], oc.U8, 0)
    s.page_table = oc.packed_tensor([1, 0], oc.I32, 0)
    check(s, [1], None)


def test_wide_spans_are_not_truncated_to_32_bits():
    s = smla(1, 32, 1)
    s.kv.shape[0] = 1 << 19
    size_to_span(s.kv)
    assert oc.wide_span(s.kv) > (1 << 33)
    check(s, [1], None)
    s.kv.capacity &= 0xFFFFFFFF
    check(s, [1], ("kv", oc.CAPACITY))


def test_dimension_boundary_is_per_axis():
    s = smla(1, 32, 1)
    s.kv.shape[0] = (1 << 31) - 1
    size_to_span(s.kv)
    check(s, [1], None)
    s.kv.shape[0] += 1
    size_to_span(s.kv)
    check(s, [1], ("kv", oc.DIMENSION))
    s = smla(1, 32, 1)
    s.page_table = oc.packed_tensor([1, (1 << 31) - 1], oc.I32, 3)
    check(s, [1], None)
    s.page_table = oc.packed_tensor([1, 1 << 31], oc.I32, 3)
    check(s, [1], ("page_table", oc.DIMENSION))


def test_arithmetic_overflow():
    s = smla(4, 32, 1)
    s.q.strides[0] = 1 << 63
    s.q.capacity = U64 - s.q.address
    check(s, [4], ("q", oc.OVERFLOW))
    s = smla(1, 32, 1)
    s.kv.strides[1] = 1 << 62
    check(s, [1], ("kv", oc.OVERFLOW))
    s = smla(1, 32, 1)
    s.q.strides[1] = 1 << 63
    check(s, [1], ("q", oc.OVERFLOW))


def test_address_end_and_capacity_are_separate():
    s = smla(1, 32, 1)
    s.q.address = U64 - s.q.capacity + 1
    check(s, [1], ("q", oc.OVERFLOW))
    s = smla(1, 32, 1)
    s.q.address = U64 - s.q.capacity - 1
    check(s, [1], None)
    s.q.capacity += 2
    check(s, [1], ("q", oc.OVERFLOW))
    s = smla(1, 32, 1)
    s.q.capacity += 1
    check(s, [1], None)


def test_output_aliases_and_adjacent_ranges():
    good = smla(4, 32, 1)
    for inp in ("q", "kv", "page_table", "seq_id", "q_pos", "kv_len"):
        s = good.copy()
        s.out.address = getattr(s, inp).address
        check(s, [4], ("out", oc.ALIAS))
        s = good.copy()
        s.lse.address = getattr(s, inp).address
        check(s, [4], ("lse", oc.ALIAS))
    s = good.copy()
    s.lse.address = s.out.address
    check(s, [4], ("lse", oc.ALIAS))
    s = good.copy()
    s.out.address = s.q.address + s.q.capacity
    check(s, [4], None)
    s.out.address -= 2
    check(s, [4], ("out", oc.ALIAS))
    s = good.copy()
    s.out.address = s.q.address - s.out.capacity
    check(s, [4], None)
    s.out.address += 2
    check(s, [4], ("out", oc.ALIAS))
    s = good.copy()
    s.q_pos.address = s.seq_id.address
    check(s, [4], None)


def test_unused_capacity_and_internal_padding():
    s = smla(1, 32, 1)
    s.out.address = s.q.address + s.q.capacity
    s.q.capacity += s.out.capacity
    check(s, [1], None)
    s = smla(2, 32, 1)
    s.q.strides[0] = 100_000
    size_to_span(s.q)
    s.lse.address = s.q.address + 40_000
    check(s, [2], ("lse", oc.ALIAS))


def test_f32_partial_output_is_accepted_and_other_dtypes_are_not():
    s = smla(2, 128, 1, oc.KV_BF16_ROPE576)
    s.out = oc.packed_tensor([2, 128, 512], oc.F32, 9)
    c = to_c(s)
    err = _abi.TqContractError()
    arr = (ctypes.c_uint8 * 1)(2)
    assert _abi.lib.tq_mla_validate(ctypes.byref(c), arr, 1, None, ctypes.byref(err)) == 0
    s.out = oc.packed_tensor([2, 128, 512], oc.I32, 9)
    c = to_c(s)
    assert _abi.lib.tq_mla_validate(ctypes.byref(c), arr, 1, None, ctypes.byref(err)) == oc.DTYPE


def test_params_are_checked_before_any_launch():
    s = smla(1, 128, 1, oc.KV_BF16_ROPE576)
    st, params = c_verdict(s, [1])
    assert st is None
    err = _abi.TqContractError()
    copy = _abi.TqMlaParams.from_buffer_copy(params)
    copy.spec.q.shape[1] = 64  # altered after validation
    assert _abi.lib.tq_mla_decode(ctypes.byref(copy), None, 0, None, ctypes.byref(err)) == 104
    assert _abi.lib.tq_mla_should_launch(ctypes.byref(copy)) == 0
    # An empty launch returns before touching any device state.
    st, empty = c_verdict(smla(0, 32, 0), [])
    assert _abi.lib.tq_mla_decode(ctypes.byref(empty), None, 0, None, ctypes.byref(err)) == 0


def test_philox_driven_boundary_sweep():
    for seed in (0, 1, 7, 42, 0xFFFFFFFF):
        for case in range(64):
            r = [int(x) for x in op.block([case, 0, 0, 0], [seed, 0])]
            counts = [x % 5 for x in r]
            tokens = sum(counts)
            s = smla(tokens, 32, 4, oc.KV_FP8_E4M3)
            stride = 528 + 16 * (r[1] % 33)
            s.kv.shape[2] = 528
            s.kv.strides = [64 * stride, stride, 1]
            s.kv.shape[0] = 1 + r[2] % 500_000
            size_to_span(s.kv)
            head_stride = 1024 + 2 * (r[3] % 99)
            s.q.strides = [32 * head_stride + 6, head_stride, 2]
            size_to_span(s.q)
            check(s, counts, None)
            if tokens > 0:
                s.kv.capacity -= 1
                check(s, counts, ("kv", oc.CAPACITY))
