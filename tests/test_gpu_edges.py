"""GPU edge cases of the reference's SMLA list (docs/TEST-PLAN.md:233-252) not covered elsewhere:
64-bit offsets in a pool over 8 GB (SMLA-E-007), extreme and degenerate logits (E-010), and two
launches running at once on two streams (E-014). All through the C ABI, against the oracle.
"""

import numpy as np
import pytest
import torch

from conftest import assert_parity
import gpu_helpers as gh
from oracle import mla as omla
from tq_mla import _abi, inputs, ops

pytestmark = pytest.mark.gpu

SCALE = 0.0625


def _np(t):
    return t.float().double().cpu().numpy()


def test_pool_over_8gb_with_rows_in_its_last_pages(cuda_device):
    """SMLA-E-007: a 1 KiB-row pool of 8.6 GB whose sequence pages are the last ones, so every
    row offset is above 2^33; dense decode and a sparse plan over the same rows."""
    pages = 131_200                                   # 131,200 x 64 x 1024 B = 8.6 GB
    kv = torch.empty((pages, 64, 512), dtype=torch.bfloat16, device=cuda_device)
    n = 4096
    # the last 64 pages, newest first; reshape keeps canonical packed strides (an inserted
    # axis would carry stride 0, which the packed-layout rule rejects)
    table = np.arange(pages - 1, pages - 1 - n // 64, -1, dtype=np.int32).reshape(1, n // 64)
    rng = np.random.default_rng(7)
    latent = torch.from_numpy(rng.standard_normal((n, 512)).astype(np.float32)).to(torch.bfloat16)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda_device)
    ops.kv_write(latent.to(cuda_device), kv, d(table), d(np.zeros(n, np.int32)),
                 d(np.arange(n, dtype=np.int32)), kv_format=_abi.KV_BF16)
    heads = 64
    q = torch.from_numpy(rng.standard_normal((1, heads, 512)).astype(np.float32)).to(torch.bfloat16)
    kv_len = np.array([n], np.int32)
    q_pos = np.array([n - 1], np.int32)
    rows_at = table[0][np.arange(n) // 64].astype(np.int64) * 64 + np.arange(n) % 64
    # the oracle sees the written rows only (an f64 copy of 8.6 GB is not needed)
    small = latent.double().numpy()
    out, lse = ops.mla_decode(q.to(cuda_device), kv, d(table), d(np.zeros(1, np.int32)),
                              d(q_pos), d(kv_len), scale=SCALE, query_counts=[1])
    torch.cuda.synchronize()
    ref_out, ref_lse = omla.identity_core(q[0].double().numpy(), small, SCALE, 512)
    assert_parity(_np(out), _np(lse), ref_out[None], ref_lse[None], label="8.6 GB pool dense")
    assert rows_at.min() * 1024 > 2 ** 33
    idx = rng.choice(n, size=2048, replace=False).astype(np.int32).reshape(1, 2048)
    out2, lse2 = ops.mla_decode(q.to(cuda_device), kv, d(table), d(np.zeros(1, np.int32)),
                                d(q_pos), d(kv_len), scale=SCALE, query_counts=[1],
                                idx=d(idx), k_len=d(np.array([2048], np.int32)))
    torch.cuda.synchronize()
    ref2, ref2_lse = omla.identity_core(q[0].double().numpy(), small[idx[0]], SCALE, 512)
    assert_parity(_np(out2), _np(lse2), ref2[None], ref2_lse[None], label="8.6 GB pool sparse")
    del kv
    torch.cuda.empty_cache()


def test_extreme_and_degenerate_logits(cuda_device):
    """SMLA-E-010: logits near +-1e5, one dominant logit, all-equal logits and subnormal inputs.
    lse is held to a relative rule at large magnitudes: f32 spacing near 1e5 is 0.008, and a
    512-term f32 score sum of terms near 1e4 rounds by ~1e-2."""
    lens = [300, 300, 300, 300]
    w = gh.workload(17, 32, lens, width=512, scale=SCALE)
    b = inputs.materialize(w, cuda_device)
    q = b.q.clone()
    q[0] *= 10000.0                     # scores of order 1e4-1e5 in both signs
    q[1] = 0
    q[1, :, 0] = 3000.0                 # one dominant direction: a few keys dominate
    q[2] = 0                            # all-equal logits
    q[3] = torch.full_like(q[3], 1e-39)  # subnormal bf16 queries
    out = torch.empty((w.tokens, w.heads, 512), dtype=torch.bfloat16, device=cuda_device)
    lse = torch.empty((w.tokens, w.heads), dtype=torch.float32, device=cuda_device)
    launch = ops.MlaLaunch(q, b.kv, b.page_table, b.seq_id, b.q_pos, b.kv_len, out, lse,
                           scale=SCALE, query_counts=b.query_counts)
    launch()
    torch.cuda.synchronize()
    assert launch.device_error() == 0
    qh, rows = gh.host_inputs(b, w)
    qh = _np(q)
    ref_out, ref_lse = omla.paged_attention(qh, rows, w.extra["page_table"], w.seq_id(),
                                            w.q_pos(), w.kv_len, scale=SCALE, value_dim=512)
    o, l_ = _np(out), lse.double().cpu().numpy()
    assert np.isfinite(o).all() and np.isfinite(l_).all()
    assert np.abs(o - ref_out).max() <= 2e-2
    assert (np.abs(l_ - ref_lse) <= 1e-3 + 1e-6 * np.abs(ref_lse)).all(), \
        np.abs(l_ - ref_lse).max()
    assert np.abs(ref_lse[0]).max() > 1e4


def test_two_launches_on_two_streams_at_once(cuda_device):
    """SMLA-E-014: two plans with their own workspaces, launched back to back on two streams
    with no synchronisation between them; each result is correct."""
    ws = [gh.workload(21, 128, [3000, 700, 64, 1500], width=576),
          gh.workload(22, 64, [129, 5000, 2048], width=576)]
    batches = [inputs.materialize(w, cuda_device) for w in ws]
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(cuda_device) for _ in ws]
    launches, outs = [], []
    for w, b in zip(ws, batches):
        out = torch.empty((w.tokens, w.heads, 512), dtype=torch.bfloat16, device=cuda_device)
        lse = torch.empty((w.tokens, w.heads), dtype=torch.float32, device=cuda_device)
        launches.append(ops.MlaLaunch(b.q, b.kv, b.page_table, b.seq_id, b.q_pos, b.kv_len, out,
                                      lse, scale=w.scale, query_counts=b.query_counts))
        outs.append((out, lse))
    for _ in range(5):
        for launch, st in zip(launches, streams):
            launch(st)
    torch.cuda.synchronize()
    for w, b, launch, (out, lse) in zip(ws, batches, launches, outs):
        assert launch.device_error() == 0
        ref_out, ref_lse = gh.oracle(b, w)
        assert_parity(_np(out), _np(lse), ref_out, ref_lse, label=f"stream {w.name}")
