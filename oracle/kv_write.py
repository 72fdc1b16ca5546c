"""Oracle (test infrastructure only): the KV cache writer, latent rows into the paged pool.

Nothing in the product imports this module; tests use it to check the CUDA writer bit for bit.

The reference plans a "latent -> 528 B KV writer" (``docs/DEV-PLAN.md:116``) over the row formats
of ``docs/HOST-CONTRACTS.md:122-123`` (1152 B bf16 latent + RoPE, 1024 B bf16 latent, 528 B FP8)
and the paged addressing of ``contracts.rs:182-209`` (position p of sequence s lives in pool row
``page_table[s][p // 64] * 64 + p % 64``). It defines no quantization rule for FP8 rows, so this
build defines one, per 128-value tile of a row (values widened exactly from bf16 to f32):

- a tile holding a NaN: scale NaN, every code 0x7F (NaN);
- otherwise amax = max |x| (possibly +inf); amax == 0: scale 0, every code 0x00;
- otherwise scale = f32(amax / 448), inv = f32(448 / amax) and code = E4M3(f32(x * inv)); when
  inv overflows to +inf (amax below ~1.3e-36) the quotient is f32(x / scale) instead. All f32
  operations round to nearest even with subnormals kept; the E4M3 conversion rounds to nearest
  even and saturates to +-448 (a NaN quotient, from inf * 0, gives 0x7F; a zero keeps its sign).

Dequantized, a code times its scale is within half an E4M3 step of x, the tile's amax maps to 448
exactly when amax / 448 is exact, and a tile of zeros reads back as zeros.
"""

import numpy as np

from oracle.fp8 import e4m3_table

PAGE_ROWS = 64
FP8_CODES = 512
FP8_PAYLOAD = 528
TILE = 128

_FINITE = e4m3_table()[:0x7F]  # codes 0x00 .. 0x7E, magnitudes increasing, 0x7E = 448


def e4m3_encode(v):
    """float32 values -> E4M3 codes (uint8): round to nearest even, saturate to +-448."""
    v = np.asarray(v, dtype=np.float32)
    nan = np.isnan(v)
    mag = np.minimum(np.abs(np.where(nan, 0.0, v)).astype(np.float64), 448.0)
    idx = np.clip(np.searchsorted(_FINITE, mag, side="right") - 1, 0, 0x7E)
    up = np.minimum(idx + 1, 0x7E)
    d_lo = mag - _FINITE[idx]
    d_hi = _FINITE[up] - mag
    take_up = (up > idx) & ((d_hi < d_lo) | ((d_hi == d_lo) & (idx % 2 == 1)))
    code = np.where(take_up, up, idx).astype(np.uint8)
    code = code | (np.signbit(v).astype(np.uint8) << 7)
    return np.where(nan, np.uint8(0x7F), code).astype(np.uint8)


def quantize_rows(x):
    """float32 ``[R, 512]`` -> (codes uint8 ``[R, 512]``, scales float32 ``[R, 4]``)."""
    x = np.asarray(x, dtype=np.float32)
    rows = x.shape[0]
    t = x.reshape(rows, 4, TILE)
    nan_tile = np.isnan(t).any(axis=2)
    amax = np.abs(np.where(np.isnan(t), np.float32(0), t)).max(axis=2).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore", under="ignore"):
        scale = (amax / np.float32(448.0)).astype(np.float32)
        inv = (np.float32(448.0) / amax).astype(np.float32)
        q_mul = (t * inv[:, :, None]).astype(np.float32)
        q_div = (t / scale[:, :, None]).astype(np.float32)
        q = np.where(np.isposinf(inv)[:, :, None], q_div, q_mul).astype(np.float32)
    codes = e4m3_encode(q)
    zero = amax == 0
    codes[zero] = 0
    scale = np.where(zero, np.float32(0), scale).astype(np.float32)
    codes[nan_tile] = 0x7F
    scale = np.where(nan_tile, np.float32(np.nan), scale).astype(np.float32)
    return codes.reshape(rows, FP8_CODES), scale


def rms_norm_rows(src_bf16_bits, weight_bf16_bits, eps):
    """RMSNorm of each row's 512 latent values with the writer's f32 arithmetic, bit for bit:
    per 16-value run the squares are added in dim order, the 32 run sums are combined pairwise at
    distances 16, 8, 4, 2, 1, mean = sum / 512, r = 1 / sqrt(mean + eps),
    y = bf16(bf16(x * r) * w), every operation an IEEE round-to-nearest f32 operation (no fused
    multiply-add). The normalised value is rounded to bf16 before the weight multiplies it, as in
    the model's RMSNorm (``self.weight * hidden_states.to(input_dtype)``, the Transformers
    ``modeling_glm5_next.py`` lines 77-81 cited by docs/reviews/2026-09-19-design-review.md:13).
    Returns the new bf16 bits (uint16 ``[R, 512]``)."""
    from oracle.fp8 import bf16_round

    f32 = np.float32
    x = (np.asarray(src_bf16_bits, dtype=np.uint16)[:, :512].astype(np.uint32) << 16).view(f32)
    w = (np.asarray(weight_bf16_bits, dtype=np.uint16).astype(np.uint32) << 16).view(f32)
    runs = x.reshape(-1, 32, 16)
    acc = np.zeros(runs.shape[:2], f32)
    with np.errstate(over="ignore", invalid="ignore", under="ignore"):
        for i in range(16):
            acc = (acc + (runs[:, :, i] * runs[:, :, i]).astype(f32)).astype(f32)
        lanes = np.arange(32)
        for o in (16, 8, 4, 2, 1):
            acc = (acc + acc[:, lanes ^ o]).astype(f32)
        total = acc[:, 0]
        r = (f32(1.0) / np.sqrt(((total / f32(512.0)).astype(f32) + f32(eps)).astype(f32))).astype(f32)
        n = bf16_round((x * r[:, None]).astype(f32)).astype(f32)
        y = (n * w[None, :]).astype(f32)
    bits = (bf16_round(y).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    nan = np.isnan(y)
    bits[nan] = 0x7FC0
    return bits


def row_bytes(src_bf16_bits, kv_format):
    """Payload bytes of each new row: ``src_bf16_bits`` is uint16 ``[R, W]`` (bf16 bit patterns).

    kv_format: 0 bf16 512 (1024 B), 1 FP8 E4M3 (528 B), 2 bf16 576 (1152 B).
    """
    src = np.ascontiguousarray(src_bf16_bits, dtype=np.uint16)
    if kv_format in (0, 2):
        return src.view(np.uint8).reshape(src.shape[0], -1)
    x = (src.astype(np.uint32) << 16).view(np.float32)
    codes, scales = quantize_rows(x)
    out = np.zeros((src.shape[0], FP8_PAYLOAD), np.uint8)
    out[:, :FP8_CODES] = codes
    out[:, FP8_CODES:] = scales.astype("<f4").view(np.uint8)
    return out


def write(pool_u8, src_bf16_bits, page_table, seq_id, pos, kv_format, norm_weight_bits=None,
          norm_eps=None):
    """Apply the writer to a copy of ``pool_u8`` (``[P, 64, r]``); returns (pool, skipped mask).

    Row t goes to ``page_table[seq_id[t]][pos[t] // 64] * 64 + pos[t] % 64``. A row whose
    sequence, position or page is out of range is skipped (the device reports it in its flags).
    When two rows name the same slot the device result is either one of them; callers do not
    write a slot twice in one call.
    """
    pool = np.array(pool_u8, copy=True)
    pages, _, stride = pool.shape
    flat = pool.reshape(pages * PAGE_ROWS, stride)
    if norm_weight_bits is not None:
        src_bf16_bits = np.array(src_bf16_bits, dtype=np.uint16, copy=True)
        src_bf16_bits[:, :512] = rms_norm_rows(src_bf16_bits, norm_weight_bits, norm_eps)
    payload = row_bytes(src_bf16_bits, kv_format)
    s_count, slots = page_table.shape
    skipped = np.zeros(len(seq_id), bool)
    for t, (s, p) in enumerate(zip(seq_id, pos)):
        s, p = int(s), int(p)
        if s < 0 or s >= s_count or p < 0 or p // PAGE_ROWS >= slots:
            skipped[t] = True
            continue
        page = int(page_table[s, p // PAGE_ROWS])
        if page < 0 or page >= pages:
            skipped[t] = True
            continue
        flat[page * PAGE_ROWS + p % PAGE_ROWS, : payload.shape[1]] = payload[t]
    return pool, skipped
