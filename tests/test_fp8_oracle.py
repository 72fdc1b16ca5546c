"""The oracle's E4M3 decoding and FP8 row dequantization (CPU).

Pinned two ways: the format's defining values (zero, the smallest subnormal, one, the largest
finite 448, the two NaN codes) and every code against PyTorch's independent float8_e4m3fn
conversion.
"""

import numpy as np
import torch

from oracle import fp8


def test_e4m3_defining_values():
    t = fp8.e4m3_table()
    assert t[0x00] == 0.0 and t[0x80] == 0.0
    assert t[0x01] == 2.0 ** -9
    assert t[0x08] == 2.0 ** -6
    assert t[0x38] == 1.0 and t[0xB8] == -1.0
    assert t[0x7E] == 448.0 and t[0xFE] == -448.0
    assert np.isnan(t[0x7F]) and np.isnan(t[0xFF])
    assert np.isfinite(np.delete(t, [0x7F, 0xFF])).all()


def test_e4m3_table_matches_torch_for_every_code():
    codes = torch.arange(256, dtype=torch.int32).to(torch.uint8)
    ref = codes.view(torch.float8_e4m3fn).to(torch.float64).numpy()
    np.testing.assert_array_equal(fp8.e4m3_table(), ref)


def test_dequant_rows_scales_each_128_tile():
    rng = np.random.default_rng(0)
    rows = np.zeros((3, 544), np.uint8)
    codes = rng.integers(0, 0x7E, size=(3, 512), dtype=np.uint8)
    scales = np.array([[0.5, 2.0, 0.125, 1.0], [1, 1, 1, 1], [3.0, 0.25, 8.0, 0.0625]], np.float32)
    rows[:, :512] = codes
    rows[:, 512:528] = scales.view(np.uint8)
    rows[:, 528:] = 0xFF  # padding past the payload is never read
    got = fp8.dequant_rows(rows)
    want = fp8.e4m3_table()[codes] * np.repeat(scales.astype(np.float64), 128, axis=1)
    np.testing.assert_array_equal(got, want)


def test_operand_rows_round_the_f32_product_to_bf16():
    rng = np.random.default_rng(1)
    rows = np.zeros((4, 528), np.uint8)
    rows[:, :512] = rng.integers(0, 0x7E, size=(4, 512), dtype=np.uint8)
    scales = rng.uniform(1e-3, 2.0, size=(4, 4)).astype(np.float32)
    rows[:, 512:528] = scales.view(np.uint8)
    codes = torch.from_numpy(rows[:, :512].copy()).view(torch.float8_e4m3fn).float()
    prod = codes * torch.from_numpy(scales).repeat_interleave(128, dim=1)
    want = prod.to(torch.bfloat16).double().numpy()
    np.testing.assert_array_equal(fp8.operand_rows(rows), want)
