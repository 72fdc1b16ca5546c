"""Oracle (test infrastructure only): pure-Python restatement of the SMLA host contract.

Nothing in the product imports this module. Tests compare the verdicts of the product's C++
validator (``tq_mla_validate``) with this restatement, case by case.

Restated from ``crates/tq-core/src/contracts.rs``:
  - ``_check``          follows ``check``            :262-325 (dtype, shape, 2**31 limit, strides,
                        then, when launching and non-empty: checked span, null address,
                        alignment, capacity, end overflow);
  - ``_check_strides``  follows ``check_strides``    :331-356;
  - ``_check_kv``       follows ``check_kv_strides`` :359-371;
  - ``_check_aliases``  follows ``check_aliases``    :407-421;
  - ``validate``        follows ``SmlaParams::new``  :437-493.
Generalisations for the dense paged path (each one is a documented extension, not a change of
the reference's rules for its own format):
  - a third row format ``BF16_ROPE576`` (576 bf16 = 1152 B: 512 latent + 64 RoPE), for which
    ``q`` is ``[T, H, 576]`` while ``out`` stays ``[T, H, 512]``;
  - heads in ``{16, 32, 64, 128}`` (the reference accepts ``{32, 64}``);
  - the softmax scale stays the exact GLM constant ``0.0625`` for the reference's 512-wide
    formats and is any finite positive ``f32`` for ``BF16_ROPE576``;
  - no sparse ``idx``/``k_len`` tensors (dense attention over ``[0, min(kv_len, q_pos+1))``);
  - ``out`` may be f32 (a partial result that a later log-sum-exp merge combines);
  - a prefill plan (``max_per_seq=None``) lifts the 4-queries-per-sequence decode limit.
"""

import math
import struct
from dataclasses import dataclass, field, replace

DIMENSION_LIMIT = 1 << 31
PAGE_ROWS = 64
KV_GRANULARITY = 16
U64 = (1 << 64) - 1
GLM_SCALE_BITS = struct.unpack("<I", struct.pack("<f", 0.0625))[0]

# Storage dtypes (values equal the C enum in include/tq_mla.h).
BF16, I32, F32, U8 = 0, 1, 2, 3
ELEMENT = {BF16: 2, I32: 4, F32: 4, U8: 1}
# Row formats.
KV_BF16, KV_FP8_E4M3, KV_BF16_ROPE576 = 0, 1, 2
PAYLOAD = {KV_BF16: 1024, KV_FP8_E4M3: 528, KV_BF16_ROPE576: 1152}
QK_WIDTH = {KV_BF16: 512, KV_FP8_E4M3: 512, KV_BF16_ROPE576: 576}
V_WIDTH = 512
HEADS = (16, 32, 64, 128)
MAX_DECODE_QUERIES = 4

SHAPE, DTYPE, DIMENSION, STRIDE, ALIGNMENT, ADDRESS, CAPACITY, OVERFLOW, QUERY_COUNT, SCALE, \
    GROUP, ALIAS = range(1, 13)
NAMES = {SHAPE: "Shape", DTYPE: "Dtype", DIMENSION: "Dimension", STRIDE: "Stride",
         ALIGNMENT: "Alignment", ADDRESS: "Address", CAPACITY: "Capacity", OVERFLOW: "Overflow",
         QUERY_COUNT: "QueryCount", SCALE: "Scale", GROUP: "Group", ALIAS: "Alias"}
FIELDS = ("q", "kv", "page_table", "seq_id", "q_pos", "kv_len", "out", "lse")


class ContractError(Exception):
    def __init__(self, field_name, kind):
        super().__init__(f"{field_name}: {NAMES[kind]}")
        self.field = field_name
        self.kind = kind


@dataclass
class Tensor:
    shape: list
    strides: list
    dtype: int
    address: int
    capacity: int


@dataclass
class Spec:
    q: Tensor
    kv: Tensor
    page_table: Tensor
    seq_id: Tensor
    q_pos: Tensor
    kv_len: Tensor
    out: Tensor
    lse: Tensor
    kv_format: int = KV_BF16_ROPE576
    scale: float = 192 ** -0.5
    extra: dict = field(default_factory=dict)

    def copy(self):
        return replace(self, **{f: replace(getattr(self, f), shape=list(getattr(self, f).shape),
                                           strides=list(getattr(self, f).strides))
                                for f in FIELDS})


def wide_span(t: Tensor) -> int:
    """Exact (unbounded) span; the test-side wide oracle of ``tests/support/mod.rs:13-24``."""
    if 0 in t.shape:
        return 0
    return ELEMENT[t.dtype] + sum((d - 1) * s for d, s in zip(t.shape, t.strides))


def packed_tensor(shape, dtype, slot):
    """Canonical packed strides and a fake numeric address ``slot << 48`` sized to the span."""
    strides = [0] * len(shape)
    stride = ELEMENT[dtype]
    for i in reversed(range(len(shape))):
        strides[i] = stride
        stride *= max(shape[i], 1)
    t = Tensor(list(shape), strides, dtype, slot << 48, 0)
    t.capacity = wide_span(t)
    return t


def _fail(name, kind):
    raise ContractError(name, kind)


def _check_strides(name, t, packed):
    el = ELEMENT[t.dtype]
    n = len(t.shape)
    if t.strides[n - 1] != el:
        _fail(name, STRIDE)
    for axis in range(n - 2, -1, -1):
        needed = t.strides[axis + 1] * max(t.shape[axis + 1], 1)
        if needed > U64:
            _fail(name, OVERFLOW)
        st = t.strides[axis]
        fits = st == needed if packed else (st >= needed and st % el == 0)
        if not fits:
            _fail(name, STRIDE)


def _check(name, t, shape, dtype, layout, launching):
    """``layout``: 'packed', 'padded' or 'rows'. Returns ``(start, end)`` or ``None``."""
    if t.dtype != dtype:
        _fail(name, DTYPE)
    if list(t.shape) != list(shape):
        _fail(name, SHAPE)
    if any(d >= DIMENSION_LIMIT for d in t.shape):
        _fail(name, DIMENSION)
    el = ELEMENT[dtype]
    if layout != "rows":
        _check_strides(name, t, layout == "packed")
    if not launching or 0 in t.shape:
        return None
    span = el
    for d, s in zip(t.shape, t.strides):
        span = span + (d - 1) * s
        if span > U64:
            _fail(name, OVERFLOW)
    if t.address == 0:
        _fail(name, ADDRESS)
    gran = KV_GRANULARITY if layout == "rows" else el
    if t.address % gran:
        _fail(name, ALIGNMENT)
    if t.capacity < span:
        _fail(name, CAPACITY)
    if t.address + t.capacity > U64:
        _fail(name, OVERFLOW)
    return (name, t.address, t.address + span)


def _check_kv(t, payload):
    row = t.strides[1]
    if t.strides[2] != 1 or row < payload or row % KV_GRANULARITY:
        _fail("kv", STRIDE)
    if PAGE_ROWS * row > U64:
        _fail("kv", OVERFLOW)
    if t.strides[0] != PAGE_ROWS * row:
        _fail("kv", STRIDE)


def _check_aliases(inputs, outputs):
    for pos, out in enumerate(outputs):
        if out is None:
            continue
        for other in list(inputs) + outputs[:pos]:
            if other is None:
                continue
            if out[1] < other[2] and other[1] < out[2]:
                _fail(out[0], ALIAS)


def _scale_ok(spec):
    """The scale as the f32 the C ABI carries (out-of-range values become infinities)."""
    import numpy as np

    with np.errstate(over="ignore"):
        f32 = np.float32(spec.scale)
    if spec.kv_format in (KV_BF16, KV_FP8_E4M3):
        return bool(np.isfinite(f32)) and int(f32.view(np.uint32)) == GLM_SCALE_BITS
    return bool(np.isfinite(f32)) and float(f32) > 0


MAX_INDICES = 2051  # contracts.rs:28


def validate(spec: Spec, query_counts, max_per_seq=MAX_DECODE_QUERIES, idx=None, k_len=None):
    """Raise ``ContractError`` for the first violation; return ``should_launch`` otherwise.

    With ``idx`` / ``k_len`` (``Tensor``) the plan is a sparse top-k plan: the index width is
    checked right after q (``contracts.rs:442-445``), idx as a padded ``[T, K]`` i32 tensor and
    k_len as a packed ``[T]`` one after kv_len (``:469-470``), and both are alias-check inputs.
    Sparse plans take the 512-wide formats of the reference (``KvFormat``, ``:127-144``).
    """
    tokens, heads, width = spec.q.shape
    sparse = idx is not None
    if spec.kv_format not in PAYLOAD:
        _fail("kv_format", SHAPE)
    if heads not in HEADS or width != QK_WIDTH[spec.kv_format]:
        _fail("q", SHAPE)
    if sparse and (k_len is None or spec.kv_format == KV_BF16_ROPE576):
        _fail("kv_format", SHAPE)
    if sparse and (len(idx.shape) != 2 or idx.shape[1] > MAX_INDICES):
        _fail("idx", SHAPE)
    if not _scale_ok(spec):
        _fail("softmax_scale", SCALE)
    sequences, slots = spec.page_table.shape
    launching = tokens != 0
    payload = PAYLOAD[spec.kv_format]
    _check_kv(spec.kv, payload)
    query = [tokens, heads, width]
    pool = [spec.kv.shape[0], PAGE_ROWS, payload]
    inputs = [
        _check("q", spec.q, query, BF16, "padded", launching),
        _check("kv", spec.kv, pool, U8, "rows", launching),
        _check("page_table", spec.page_table, [sequences, slots], I32, "packed", launching),
        _check("seq_id", spec.seq_id, [tokens], I32, "packed", launching),
        _check("q_pos", spec.q_pos, [tokens], I32, "packed", launching),
        _check("kv_len", spec.kv_len, [sequences], I32, "packed", launching),
    ]
    if sparse:
        inputs += [
            _check("idx", idx, [tokens, idx.shape[1]], I32, "padded", launching),
            _check("k_len", k_len, [tokens], I32, "packed", launching),
        ]
    outputs = [
        _check("out", spec.out, [tokens, heads, V_WIDTH], F32 if spec.out.dtype == F32 else BF16,
               "padded", launching),
        _check("lse", spec.lse, [tokens, heads], F32, "packed", launching),
    ]
    if len(query_counts) != sequences:
        _fail("query_counts", QUERY_COUNT)
    planned = 0
    for c in query_counts:
        if max_per_seq is not None and c > max_per_seq:
            _fail("query_counts", QUERY_COUNT)
        planned += c
    if planned != tokens:
        _fail("query_counts", QUERY_COUNT)
    _check_aliases(inputs, outputs)
    return launching


def make_spec(tokens, heads, sequences, *, kv_format=KV_BF16_ROPE576, pages=17, slots=16,
              scale=None):
    """A valid spec with fake addresses, in the style of ``tests/support/mod.rs:48-63``."""
    width = QK_WIDTH[kv_format]
    payload = PAYLOAD[kv_format]
    if scale is None:
        scale = 0.0625 if kv_format != KV_BF16_ROPE576 else 192 ** -0.5
    return Spec(
        q=packed_tensor([tokens, heads, width], BF16, 1),
        kv=packed_tensor([pages, PAGE_ROWS, payload], U8, 2),
        page_table=packed_tensor([sequences, slots], I32, 3),
        seq_id=packed_tensor([tokens], I32, 4),
        q_pos=packed_tensor([tokens], I32, 5),
        kv_len=packed_tensor([sequences], I32, 6),
        out=packed_tensor([tokens, heads, V_WIDTH], BF16, 9),
        lse=packed_tensor([tokens, heads], F32, 10),
        kv_format=kv_format,
        scale=scale,
    )
