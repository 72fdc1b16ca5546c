"""GPU: one attention layer's step through the C ABI, prologue then attention, against the
oracle's chain (prologue oracle, writer oracle, paged attention oracle).

Every token of each sequence goes through ``tq_mla_prologue`` (its row lands in the paged pool),
then the last token of each sequence attends over its whole sequence with ``tq_mla_decode``.
The reference's no-RoPE model sizes (hidden 4096, Q rank 1536, 64 heads of 256, scale 256^-0.5)
with bf16 and FP8 rows; the 576-wide RoPE form with 128 heads. The attention step is checked on
the prologue's own output at the attention path's tolerances, and the whole chain against the
oracle chain with an lse bound that covers the spread of q (``assert_parity``)."""

import numpy as np
import pytest
import torch

from conftest import assert_parity
from oracle import fp8 as ofp8
from oracle import mla as omla
from oracle import prologue as opro
from tq_mla import _abi, ops

pytestmark = pytest.mark.gpu

ROW = {_abi.KV_BF16: 1024, _abi.KV_FP8_E4M3: 544, _abi.KV_BF16_ROPE576: 1152}


def _bf16(a, device):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16).to(device)


@pytest.mark.parametrize("fmt,heads,dn,dr,dm", [(_abi.KV_BF16, 64, 256, 0, 4096),
                                                (_abi.KV_FP8_E4M3, 64, 256, 0, 4096),
                                                (_abi.KV_BF16_ROPE576, 128, 128, 64, 2048)])
def test_prologue_then_decode_matches_the_oracle_chain(cuda_device, fmt, heads, dn, dr, dm):
    rng = np.random.default_rng(31 + fmt)
    rq = 1536
    lens = rng.integers(65, 400, 6)
    lens[0] = 64                                   # one sequence ends on a page boundary
    seqs, slots = len(lens), 8
    table = rng.permutation(seqs * slots).astype(np.int32).reshape(seqs, slots)
    seq = np.concatenate([np.full(n, b, np.int32) for b, n in enumerate(lens)])
    pos = np.concatenate([np.arange(n, dtype=np.int32) for n in lens])
    w = dict(x=rng.standard_normal((len(seq), dm)),
             w_qa=rng.standard_normal((rq, dm)) / np.sqrt(dm),
             q_norm=rng.uniform(0.5, 1.5, rq),
             w_qb=rng.standard_normal((heads * (dn + dr), rq)) / np.sqrt(rq),
             w_uk=rng.standard_normal((heads, dn, 512)) / np.sqrt(dn),
             w_kva=rng.standard_normal((512 + dr, dm)) / np.sqrt(dm),
             kv_norm=rng.uniform(0.5, 1.5, 512))
    dev = {k: _bf16(v, cuda_device) for k, v in w.items()}
    host = {k: v.float().cpu().numpy().astype(np.float64) for k, v in dev.items()}
    pool = torch.zeros((seqs * slots, 64, ROW[fmt]), dtype=torch.uint8, device=cuda_device)
    d_table = torch.from_numpy(table).to(cuda_device)
    d_pos = torch.from_numpy(pos).to(cuda_device)
    flags = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    q_all = ops.mla_prologue(dev["x"], dev["w_qa"], dev["q_norm"], dev["w_qb"], dev["w_uk"],
                             dev["w_kva"], dev["kv_norm"], d_pos, torch.from_numpy(seq).to(cuda_device),
                             d_table, pool, heads=heads, nope_dim=dn, rope_dim=dr, kv_format=fmt,
                             flags=flags)
    last = np.cumsum(lens) - 1
    q = q_all[torch.from_numpy(last).to(cuda_device)].contiguous()
    kv_len = lens.astype(np.int32)
    scale = 0.0625 if dr == 0 else 192 ** -0.5
    out, lse = ops.mla_decode(q, pool, d_table, torch.arange(seqs, dtype=torch.int32,
                                                             device=cuda_device),
                              torch.from_numpy(kv_len - 1).to(cuda_device),
                              torch.from_numpy(kv_len).to(cuda_device), scale=scale,
                              query_counts=[1] * seqs, kv_format=fmt)
    torch.cuda.synchronize()
    assert int(flags.item()) == 0
    # the oracle's chain: queries of the last tokens, rows of every token, then attention
    q_ref, _ = opro.prologue(host["x"][last], host["w_qa"], host["q_norm"], host["w_qb"],
                             host["w_uk"], host["w_kva"], host["kv_norm"], pos[last], heads=heads,
                             nope_dim=dn, rope_dim=dr, q_eps=1e-6, kv_eps=1e-6, rope_theta=10000.0)
    kvf = opro.cache_rows(host["x"], host["w_kva"], pos, rope_dim=dr, rope_theta=10000.0)
    pool_ref, skipped = opro.write_rows(np.zeros(tuple(pool.shape), np.uint8), kvf,
                                        host["kv_norm"], table, seq, pos, kv_format=fmt,
                                        kv_eps=1e-6)
    assert not skipped.any()
    flat = pool_ref.reshape(-1, ROW[fmt])
    if fmt == _abi.KV_FP8_E4M3:
        rows = ofp8.operand_rows(flat)
    else:
        rows = (flat.copy().view(np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    got_out, got_lse = out.double().cpu().numpy(), lse.double().cpu().numpy()
    # 1. the attention step on exactly what the prologue produced (its q, the pool it wrote):
    #    the attention path's own tolerances
    pool_np = pool.cpu().numpy().reshape(-1, ROW[fmt])
    if fmt == _abi.KV_FP8_E4M3:
        own_rows = ofp8.operand_rows(pool_np)
    else:
        own_rows = (pool_np.copy().view(np.uint16).astype(np.uint32) << 16).view(
            np.float32).astype(np.float64)
    own_out, own_lse = omla.paged_attention(q.double().cpu().numpy(), own_rows, table,
                                            np.arange(seqs), kv_len - 1, kv_len, scale=scale,
                                            value_dim=512)
    assert_parity(got_out, got_lse, own_out, own_lse, label=f"decode on the prologue's output ({fmt})")
    # 2. the whole chain against the oracle chain: q differs from the float64 oracle's by bf16
    #    rounding propagated through the projections (relative L2 ~2^-8), which moves the scores
    #    and so lse by up to a few 1e-3. FP8 rows: a projected value one bf16 step away can land
    #    one E4M3 step away (up to 12.5% of the value; 1-3% of the codes), so the outputs get
    #    3x the attention path's bounds there.
    ref_out, ref_lse = omla.paged_attention(q_ref, rows, table, np.arange(seqs), kv_len - 1,
                                            kv_len, scale=scale, value_dim=512)
    wide = 3.0 if fmt == _abi.KV_FP8_E4M3 else 1.0
    assert_parity(got_out, got_lse, ref_out, ref_lse, label=f"prologue -> decode ({fmt})",
                  lse_abs=5e-3, out_abs=wide * 2e-2, out_rel=wide * 1e-2)
