"""Oracle (test infrastructure only): FP8 E4M3 KV rows decoded in float64.

Nothing in the product imports this module; tests use it to check the CUDA kernels.

Row format (``docs/HOST-CONTRACTS.md:122-123``, ``docs/TEST-PLAN.md:181-184``): bytes 0-511 hold
512 E4M3 codes, bytes 512-527 hold four little-endian f32 scales, one per 128 values; the cached
latent value is ``e4m3(code[i]) * scale[i // 128]``. E4M3 here is the OCP FP8 format named by the
contract: 1 sign bit, 4 exponent bits with bias 7, 3 mantissa bits, subnormals, no infinities,
and NaN only for exponent and mantissa all ones (0x7F, 0xFF); the largest finite magnitude is 448.
"""

import numpy as np

ROW_CODES = 512
ROW_PAYLOAD = 528
TILE = 128


def e4m3_table():
    """float64 value of each of the 256 codes (NaN for 0x7F and 0xFF)."""
    c = np.arange(256)
    sign = np.where(c >> 7, -1.0, 1.0)
    e = (c >> 3) & 15
    m = (c & 7).astype(np.float64)
    mag = np.where(e == 0, m / 8.0 * 2.0 ** -6, (1.0 + m / 8.0) * 2.0 ** (e.astype(np.float64) - 7))
    mag = np.where((e == 15) & (m == 7), np.nan, mag)
    return sign * mag


_TABLE = e4m3_table()


def dequant_rows(rows_u8):
    """``uint8 [R, >=528]`` FP8 rows -> float64 ``[R, 512]`` latent values."""
    rows_u8 = np.ascontiguousarray(rows_u8[:, :ROW_PAYLOAD])
    codes = rows_u8[:, :ROW_CODES]
    scales = rows_u8[:, ROW_CODES:ROW_PAYLOAD].copy().view("<f4").astype(np.float64)
    return _TABLE[codes] * np.repeat(scales, TILE, axis=1)


def bf16_round(x):
    """float32 values rounded to the nearest bfloat16 (ties to even), returned as float64."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    out = (r & 0xFFFFFFFF).astype(np.uint32).view(np.float32).astype(np.float64)
    out[nan] = np.nan
    return out


def operand_rows(rows_u8):
    """The latent values as a bf16 tensor-core operand: ``e4m3(code) * scale`` computed in f32
    (the code is exact in f32) and rounded once to bf16. Kernels that dequantize into bf16 shared
    memory compute on these; comparing them with the oracle on these values separates the one
    operand rounding from the rest of the arithmetic."""
    rows_u8 = np.ascontiguousarray(rows_u8[:, :ROW_PAYLOAD])
    codes = _TABLE[rows_u8[:, :ROW_CODES]].astype(np.float32)
    scales = rows_u8[:, ROW_CODES:ROW_PAYLOAD].copy().view("<f4")
    with np.errstate(invalid="ignore", over="ignore"):
        prod = codes * np.repeat(scales, TILE, axis=1)
    return bf16_round(prod)
