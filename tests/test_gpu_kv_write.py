"""GPU: the KV cache writer (tq_kv_write) through the C ABI, bit for bit against the oracle.

The whole pool is compared byte for byte, rows the call did not name and the padding past each
row's payload included. Special tiles exercise every branch of the FP8 rule: zeros, a NaN, an
infinity, subnormal magnitudes, values that round to signed zero, and saturation at 448.
"""

import numpy as np
import pytest
import torch

from conftest import assert_parity
from oracle import fp8 as ofp8
from oracle import kv_write as okw
from oracle import mla as omla
from tq_mla import _abi, ops

pytestmark = pytest.mark.gpu

WIDTH = {_abi.KV_BF16: 512, _abi.KV_FP8_E4M3: 512, _abi.KV_BF16_ROPE576: 576}
PAYLOAD = {_abi.KV_BF16: 1024, _abi.KV_FP8_E4M3: 528, _abi.KV_BF16_ROPE576: 1152}


def _src_rows(rng, rows, width):
    x = (rng.standard_normal((rows, width)) * np.exp(rng.uniform(-6, 6, (rows, 1)))).astype(np.float32)
    if rows >= 8 and width == 512:
        x[0, 0:128] = 0.0                                 # zero tile
        x[0, 128:256] = -0.0
        x[1, 130] = np.nan                                # NaN tile
        x[2, 300] = np.inf                                # inf tile: quotients 0 and NaN
        x[2, 301] = -np.inf
        x[3, :128] = rng.standard_normal(128) * 1e-39     # subnormal magnitudes
        x[4, :128] = rng.standard_normal(128) * 1e-3
        x[4, 5] = 1e3                                     # small values round to signed zero
        x[5, 384:512] = 448.0                             # exact amax step
        x[5, 400] = -448.0
    return torch.from_numpy(x).to(torch.bfloat16)


def _case(seed, fmt, row_stride, rows, seqs=6, slots=40, pages=None, device="cuda"):
    rng = np.random.default_rng(seed)
    pages = pages or seqs * slots
    pool = torch.from_numpy(rng.integers(0, 256, size=(pages, 64, row_stride), dtype=np.uint8))
    table = rng.permutation(pages).astype(np.int32)[: seqs * slots].reshape(seqs, slots)
    # distinct (sequence, position) slots
    flat = rng.choice(seqs * slots * 64, size=rows, replace=False)
    seq_id = (flat // (slots * 64)).astype(np.int32)
    pos = (flat % (slots * 64)).astype(np.int32)
    src = _src_rows(rng, rows, WIDTH[fmt])
    return pool, table, seq_id, pos, src


def _run(pool, table, seq_id, pos, src, fmt, device, src_pad=0, flags=True):
    d_pool = pool.to(device)
    width = src.shape[1]
    if src_pad:
        big = torch.zeros((src.shape[0], width + src_pad), dtype=torch.bfloat16, device=device)
        big[:, :width] = src.to(device)
        d_src = big[:, :width]
    else:
        d_src = src.to(device)
    d_flags = torch.zeros(1, dtype=torch.int32, device=device) if flags else None
    ops.kv_write(d_src, d_pool, torch.from_numpy(table).to(device),
                 torch.from_numpy(seq_id).to(device), torch.from_numpy(pos).to(device),
                 kv_format=fmt, flags=d_flags)
    torch.cuda.synchronize()
    return d_pool.cpu().numpy(), (int(d_flags.item()) if flags else 0)


@pytest.mark.parametrize("fmt,row_stride", [
    (_abi.KV_FP8_E4M3, 544), (_abi.KV_FP8_E4M3, 528),
    (_abi.KV_BF16, 1024), (_abi.KV_BF16_ROPE576, 1152), (_abi.KV_BF16_ROPE576, 1168),
])
def test_writer_matches_the_oracle_bit_for_bit(cuda_device, fmt, row_stride):
    pool, table, seq_id, pos, src = _case(11 + fmt, fmt, row_stride, rows=3000)
    got, flags = _run(pool, table, seq_id, pos, src, fmt, cuda_device, src_pad=64)
    bits = src.view(torch.int16).numpy().view(np.uint16)
    want, skipped = okw.write(pool.numpy(), bits, table, seq_id, pos, fmt)
    assert flags == 0 and not skipped.any()
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("fmt,row_stride", [
    (_abi.KV_FP8_E4M3, 544), (_abi.KV_BF16, 1024), (_abi.KV_BF16_ROPE576, 1152),
])
def test_writer_with_rms_norm_matches_the_oracle_bit_for_bit(cuda_device, fmt, row_stride):
    """The optional RMSNorm before the write: the oracle restates the kernel's f32 operation order,
    so every byte of the pool matches (the 64 RoPE values of a 576-wide row are copied)."""
    pool, table, seq_id, pos, src = _case(31 + fmt, fmt, row_stride, rows=2000)
    src = src.clone()
    src[:16] = torch.randn((16, src.shape[1])).to(torch.bfloat16)  # no NaN or inf rows
    src[16:] = torch.nan_to_num(src[16:].float(), nan=0.0, posinf=1.0,
                                neginf=-1.0).to(torch.bfloat16)
    rng = np.random.default_rng(fmt)
    weight = torch.from_numpy(rng.uniform(0.25, 2.0, 512).astype(np.float32)).to(torch.bfloat16)
    d_pool = pool.to(cuda_device)
    flags = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ops.kv_write(src.to(cuda_device), d_pool, torch.from_numpy(table).to(cuda_device),
                 torch.from_numpy(seq_id).to(cuda_device), torch.from_numpy(pos).to(cuda_device),
                 kv_format=fmt, flags=flags, norm_weight=weight.to(cuda_device), norm_eps=1e-6)
    torch.cuda.synchronize()
    bits = src.view(torch.int16).numpy().view(np.uint16)
    wbits = weight.view(torch.int16).numpy().view(np.uint16)
    want, skipped = okw.write(pool.numpy(), bits, table, seq_id, pos, fmt,
                              norm_weight_bits=wbits, norm_eps=1e-6)
    assert int(flags.item()) == 0 and not skipped.any()
    np.testing.assert_array_equal(d_pool.cpu().numpy(), want)


def test_fp8_special_tiles_land_as_defined(cuda_device):
    pool, table, seq_id, pos, src = _case(5, _abi.KV_FP8_E4M3, 544, rows=8)
    got, _ = _run(pool, table, seq_id, pos, src, _abi.KV_FP8_E4M3, cuda_device)
    rows = got.reshape(-1, 544)
    slot = lambda t: int(table[seq_id[t], pos[t] // 64]) * 64 + int(pos[t]) % 64
    sc = lambda t: rows[slot(t), 512:528].copy().view("<f4")
    assert sc(0)[0] == 0 and sc(0)[1] == 0 and (rows[slot(0), :256] == 0).all()
    assert np.isnan(sc(1)[1]) and (rows[slot(1), 128:256] == 0x7F).all()
    assert np.isinf(sc(2)[2]) and rows[slot(2), 300] == 0x7F and rows[slot(2), 301] == 0x7F
    assert 0 < sc(3)[0] < 1.2e-38                       # a subnormal scale, kept
    assert rows[slot(5), 384] == 0x7E and rows[slot(5), 400] == 0xFE and sc(5)[3] == 1.0


def test_out_of_range_rows_are_skipped_and_flagged(cuda_device):
    pool, table, seq_id, pos, src = _case(7, _abi.KV_FP8_E4M3, 544, rows=64)
    table[2, 3] = -1
    table[4, 0] = 10 ** 6
    seq_id[5], pos[6] = 99, 40 * 64            # bad sequence; position past the table
    seq_id[7], pos[7] = 2, 3 * 64 + 9          # page entry -1
    seq_id[8], pos[8] = 4, 17                  # page entry past the pool
    got, flags = _run(pool, table, seq_id, pos, src, _abi.KV_FP8_E4M3, cuda_device)
    bits = src.view(torch.int16).numpy().view(np.uint16)
    want, skipped = okw.write(pool.numpy(), bits, table, seq_id, pos, _abi.KV_FP8_E4M3)
    assert skipped.sum() >= 4
    assert flags == (_abi.DEV_SEQ_RANGE | _abi.DEV_TABLE_SHORT | _abi.DEV_PAGE_RANGE)
    np.testing.assert_array_equal(got, want)


def test_written_fp8_rows_feed_the_attention_kernel(cuda_device):
    """Write a cache through the writer, then attend over it: the FP8 kernel against the oracle
    on the dequantized pool (the writer's rows are the kernel's input format)."""
    rng = np.random.default_rng(21)
    lens = [700, 64, 1500, 129]
    seqs, slots = len(lens), 24
    pages = seqs * slots
    table = rng.permutation(pages).astype(np.int32).reshape(seqs, slots)
    seq_id = np.concatenate([np.full(n, b, np.int32) for b, n in enumerate(lens)])
    pos = np.concatenate([np.arange(n, dtype=np.int32) for n in lens])
    latent = torch.from_numpy(rng.standard_normal((len(pos), 512)).astype(np.float32)).to(torch.bfloat16)
    pool = torch.zeros((pages, 64, 544), dtype=torch.uint8)
    pool_np, flags = _run(pool, table, seq_id, pos, latent, _abi.KV_FP8_E4M3, cuda_device)
    assert flags == 0
    d_pool = torch.from_numpy(pool_np).to(cuda_device)
    heads = 128
    q = torch.from_numpy(rng.standard_normal((seqs, heads, 512)).astype(np.float32)).to(torch.bfloat16)
    kv_len = np.array(lens, np.int32)
    q_pos = kv_len - 1
    out = torch.empty((seqs, heads, 512), dtype=torch.bfloat16, device=cuda_device)
    lse = torch.empty((seqs, heads), dtype=torch.float32, device=cuda_device)
    ops.mla_decode(q.to(cuda_device), d_pool, torch.from_numpy(table).to(cuda_device),
                   torch.arange(seqs, dtype=torch.int32, device=cuda_device),
                   torch.from_numpy(q_pos).to(cuda_device), torch.from_numpy(kv_len).to(cuda_device),
                   scale=0.0625, query_counts=[1] * seqs, out=out, lse=lse,
                   kv_format=_abi.KV_FP8_E4M3)
    torch.cuda.synchronize()
    rows = ofp8.operand_rows(pool_np.reshape(-1, 544))
    ref_out, ref_lse = omla.paged_attention(q.double().numpy(), rows, table, np.arange(seqs),
                                            q_pos, kv_len, scale=0.0625, value_dim=512)
    assert_parity(out.float().double().cpu().numpy(), lse.double().cpu().numpy(), ref_out,
                  ref_lse, label="writer -> fp8 decode")
