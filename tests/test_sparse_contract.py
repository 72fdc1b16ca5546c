"""Host contract of sparse top-k plans (tq_mla_sparse_validate), CPU only.

The index tensors follow SmlaParams::new (crates/tq-core/src/contracts.rs:442-470): the index
width above 2051 is rejected right after q, idx is checked as a padded [T, K] i32 tensor and k_len
as a packed [T] i32 tensor after kv_len, and both take part in the alias check. Fake numeric
addresses (slot << 48) as in the dense contract tests. Every verdict of the C validator is
compared with the oracle restatement (oracle/contracts.py validate with idx / k_len).
"""

import ctypes

import pytest

from oracle import contracts as oc
from test_contracts import smla, to_c
from tq_mla import _abi

SHAPE, DTYPE, STRIDE, ADDRESS, CAPACITY, QUERY_COUNT, ALIAS = 1, 2, 4, 6, 7, 9, 12
I32 = _abi.DTYPE_I32


class T:
    """An oracle tensor declaration whose fields can be edited like the C struct's."""

    def __init__(self, shape, strides, slot):
        self.o = oc.Tensor(list(shape), list(strides), oc.I32, slot << 48, 0)
        self.o.capacity = oc.wide_span(self.o)

    def c(self):
        t = _abi.TqTensorSpec()
        t.rank = len(self.o.shape)
        for i, (d, st) in enumerate(zip(self.o.shape, self.o.strides)):
            t.shape[i], t.strides_bytes[i] = d & U64, st & U64
        t.dtype = self.o.dtype
        t.device_address = self.o.address & U64
        t.buffer_bytes = self.o.capacity & U64
        return t


U64 = (1 << 64) - 1


def verdict(spec, idx, k_len, counts):
    """The C verdict (field, kind) or None, after checking the oracle gives the same one."""
    c = to_c(spec)
    params = _abi.TqMlaParams()
    err = _abi.TqContractError()
    arr = (ctypes.c_uint8 * max(1, len(counts)))(*[x & 0xFF for x in counts])
    ci, ck = idx.c(), k_len.c()
    st = _abi.lib.tq_mla_sparse_validate(ctypes.byref(c), ctypes.byref(ci), ctypes.byref(ck),
                                         arr, len(counts), ctypes.byref(params),
                                         ctypes.byref(err))
    cv = None if st == 0 else (err.field.decode(), st)
    try:
        oc.validate(spec, counts, idx=idx.o, k_len=k_len.o)
        ov = None
    except oc.ContractError as e:
        ov = (e.field, e.kind)
    assert cv == ov, (cv, ov)
    return cv, params


def case(counts=(1, 2, 4), heads=32, k=2048, fmt=oc.KV_BF16, idx_row=None):
    t = sum(counts)
    spec = smla(t, heads, len(counts), fmt)
    idx = T([t, k], [idx_row or 4 * max(k, 1), 4], 40)  # canonical empty stride for K = 0
    k_len = T([t], [4], 41)
    return spec, idx, k_len, list(counts)


@pytest.mark.parametrize("fmt", [oc.KV_BF16, oc.KV_FP8_E4M3])
@pytest.mark.parametrize("k", [0, 1, 64, 2051])
def test_accepted_plans_carry_the_index_tensors(fmt, k):
    spec, idx, k_len, counts = case(k=k, fmt=fmt)
    v, params = verdict(spec, idx, k_len, counts)
    assert v is None
    assert params.sparse == 1 and params.topk == k and params.should_launch == 1
    assert params.idx.shape[1] == k and params.k_len.shape[0] == sum(counts)
    assert _abi.lib.tq_mla_should_launch(ctypes.byref(params)) == 1
    params.topk += 1  # a modified plan is refused by the digest
    assert _abi.lib.tq_mla_should_launch(ctypes.byref(params)) == 0


def test_padded_index_rows_are_allowed():
    spec, idx, k_len, counts = case(k=100, idx_row=4 * 128)
    assert verdict(spec, idx, k_len, counts)[0] is None


def test_rejections():
    spec, idx, k_len, counts = case(k=2052)
    assert verdict(spec, idx, k_len, counts)[0] == ("idx", SHAPE)
    spec, idx, k_len, counts = case(fmt=oc.KV_BF16_ROPE576)
    assert verdict(spec, idx, k_len, counts)[0] == ("kv_format", SHAPE)
    spec, idx, k_len, counts = case()
    idx.o.dtype = oc.F32
    assert verdict(spec, idx, k_len, counts)[0] == ("idx", DTYPE)
    spec, idx, k_len, counts = case()
    idx.o.shape[0] -= 1
    assert verdict(spec, idx, k_len, counts)[0] == ("idx", SHAPE)
    spec, idx, k_len, counts = case(idx_row=4 * 2048 + 2)
    assert verdict(spec, idx, k_len, counts)[0] == ("idx", STRIDE)
    spec, idx, k_len, counts = case()
    k_len.o.strides[0] = 8
    assert verdict(spec, idx, k_len, counts)[0] == ("k_len", STRIDE)
    spec, idx, k_len, counts = case()
    k_len.o.address = 0
    assert verdict(spec, idx, k_len, counts)[0] == ("k_len", ADDRESS)
    spec, idx, k_len, counts = case()
    idx.o.capacity -= 1
    assert verdict(spec, idx, k_len, counts)[0] == ("idx", CAPACITY)
    spec, idx, k_len, counts = case(counts=(5,))
    assert verdict(spec, idx, k_len, counts)[0] == ("query_counts", QUERY_COUNT)
    spec, idx, k_len, counts = case(heads=48)
    assert verdict(spec, idx, k_len, counts)[0] == ("q", SHAPE)


def test_index_tensors_take_part_in_the_alias_check():
    spec, idx, k_len, counts = case()
    idx.o.address = spec.out.address + 64
    assert verdict(spec, idx, k_len, counts)[0] == ("out", ALIAS)


def test_empty_batch_needs_no_index_storage():
    spec, idx, k_len, counts = case(counts=(0, 0))
    for t in (idx, k_len):
        t.o.address = 0
        t.o.capacity = 0
    v, params = verdict(spec, idx, k_len, counts)
    assert v is None and params.should_launch == 0
