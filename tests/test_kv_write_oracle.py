"""The KV writer oracle (CPU): E4M3 encoding pinned against PyTorch, the tile scale rule, and
the paged scatter."""

import numpy as np
import torch

from oracle import fp8 as ofp8
from oracle import kv_write as okw


def test_e4m3_encode_matches_torch_rne_inside_the_range():
    rng = np.random.default_rng(0)
    v = np.concatenate([rng.standard_normal(20000) * 50, rng.uniform(-448, 448, 20000),
                        rng.standard_normal(5000) * 2.0 ** -8, ofp8.e4m3_table()[:0x7F],
                        # exact midpoints between neighbouring codes (ties to even)
                        (ofp8.e4m3_table()[1:0x7F] + ofp8.e4m3_table()[:0x7E]) / 2]).astype(np.float32)
    v = np.concatenate([v, -v])
    want = torch.from_numpy(v).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(okw.e4m3_encode(v), want)


def test_e4m3_encode_saturates_and_keeps_signs():
    v = np.array([448.0, 449.0, 464.0, 1e30, np.inf, -np.inf, -0.0, 0.0, -1e-9, np.nan], np.float32)
    got = okw.e4m3_encode(v)
    assert got.tolist() == [0x7E, 0x7E, 0x7E, 0x7E, 0x7E, 0xFE, 0x80, 0x00, 0x80, 0x7F]


def test_quantize_rows_tile_rules():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((5, 512)).astype(np.float32)
    x[1, 128:256] = 0.0                     # zero tile
    x[2, 0:128] = np.float32(1e-40)         # subnormal amax
    x[3, 300] = np.nan                      # NaN tile
    x[4, 400] = np.inf                      # inf tile
    codes, scales = okw.quantize_rows(x)
    assert scales[1, 1] == 0 and (codes[1, 128:256] == 0).all()
    assert np.isnan(scales[3, 2]) and (codes[3, 256:384] == 0x7F).all()
    assert np.isinf(scales[4, 3]) and codes[4, 400] == 0x7F
    assert set(codes[4, 384:512][np.arange(128) != 16].tolist()) <= {0x00, 0x80}
    # ordinary tiles: each tile's amax maps to +-448 and every value within half a step
    ok = np.isfinite(scales) & (scales > 0)
    with np.errstate(invalid="ignore"):
        deq = ofp8.e4m3_table()[codes].reshape(5, 4, 128) * scales[:, :, None]
        err = np.abs(deq - x.reshape(5, 4, 128))
    # half an E4M3 step: 2^-4 relative for normals, 2^-10 * scale in the subnormal range
    bound = np.maximum(np.abs(x.reshape(5, 4, 128)) * 2.0 ** -4, scales[:, :, None] * 2.0 ** -10)
    assert (err <= bound)[ok].all()
    assert (np.abs(codes.reshape(5, 4, 128)[0]) & 0x7F).max() == 0x7E


def test_write_scatters_rows_and_skips_bad_slots():
    rng = np.random.default_rng(2)
    pool = rng.integers(0, 256, size=(6, 64, 544), dtype=np.uint8)
    table = np.array([[4, 1, -1], [0, 5, 2]], np.int32)
    seq_id = np.array([0, 1, 1, 0, 2, 0], np.int32)
    pos = np.array([70, 3, 150, 130, 1, 200], np.int32)
    src = rng.standard_normal((6, 512)).astype(np.float32)
    bits = (src.view(np.uint32) >> 16).astype(np.uint16)
    new, skipped = okw.write(pool, bits, table, seq_id, pos, 1)
    assert skipped.tolist() == [False, False, False, True, True, True]
    rows = new.reshape(-1, 544)
    payload = okw.row_bytes(bits, 1)
    assert (rows[1 * 64 + 6, :528] == payload[0]).all()
    assert (rows[0 * 64 + 3, :528] == payload[1]).all()
    assert (rows[2 * 64 + 22, :528] == payload[2]).all()
    changed = np.flatnonzero((new != pool).any(axis=2).reshape(-1))
    assert set(changed.tolist()) <= {70, 3, 150}
    assert (new.reshape(-1, 544)[:, 528:] == pool.reshape(-1, 544)[:, 528:]).all()


def test_rms_norm_rows_is_rmsnorm_to_bf16_rounding():
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((6, 512)) * np.exp(rng.uniform(-8, 8, (6, 1)))).astype(np.float32)
    w = rng.uniform(0.5, 1.5, 512).astype(np.float32)
    bits = lambda a: (torch.from_numpy(a).to(torch.bfloat16).view(torch.int16).numpy()
                      .view(np.uint16))
    xb, wb = bits(x), bits(w)
    got = (okw.rms_norm_rows(xb, wb, 1e-6).astype(np.uint32) << 16).view(np.float32)
    xf = (xb.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    wf = (wb.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    want = xf / np.sqrt((xf ** 2).mean(axis=1, keepdims=True) + 1e-6) * wf
    np.testing.assert_allclose(got, want, rtol=2 ** -7, atol=1e-30)
    # the rounding points of the model's RMSNorm: bf16(w * bf16(x * r)), x * r in f32
    r = (1.0 / np.sqrt((xf ** 2).mean(axis=1, keepdims=True) + 1e-6)).astype(np.float32)
    n = ofp8.bf16_round((xf.astype(np.float32) * r).astype(np.float32)).astype(np.float32)
    twice = ofp8.bf16_round((n * wf.astype(np.float32)).astype(np.float32))
    assert np.mean(got == twice) > 0.99
