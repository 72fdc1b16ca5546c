"""GPU device-side error flags (read back with tq_mla_read_device_error).

The launch grid never depends on the data, so bad metadata cannot be rejected on the host
without a device read; the kernels instead check it and flag it (include/tq_mla.h):
  - a page-table entry outside [0, pages): that page is fetched entirely out of bounds, which
    the TMA fills with zeros, so no pool byte outside the pool is read (docs/TEST-PLAN.md:
    "masked lanes never dereference the pool");
  - a seq_id outside [0, sequences): the token is left with no visible key (zeros, lse -inf);
  - a kv_len beyond 64 x the page-table width: clamped to the table.
Tokens whose own metadata is valid are unaffected and still match the oracle.
"""

import numpy as np
import pytest
import torch

from conftest import assert_parity
import gpu_helpers as gh
from tq_mla import inputs, ops

pytestmark = pytest.mark.gpu

PAGE_RANGE, SEQ_RANGE, TABLE_SHORT = 2, 4, 8


def _np(t):
    return t.float().double().cpu().numpy()


def _launch(b, w):
    out = torch.empty((w.tokens, w.heads, 512), dtype=torch.bfloat16, device=b.q.device)
    lse = torch.empty((w.tokens, w.heads), dtype=torch.float32, device=b.q.device)
    launch = ops.MlaLaunch(b.q, b.kv, b.page_table, b.seq_id, b.q_pos, b.kv_len, out, lse,
                           scale=w.scale, query_counts=b.query_counts)
    launch()
    torch.cuda.synchronize()
    return launch.device_error(), _np(out), _np(lse)


def test_page_index_outside_pool(cuda_device):
    w = gh.workload(41, 128, [200, 300, 129])
    b = inputs.materialize(w, cuda_device)
    pt = b.page_table.clone()
    pt[0, 0] = -1                 # negative
    pt[1, 1] = w.pool_pages + 5   # past the pool
    b.page_table.copy_(pt)
    flags, out, lse = _launch(b, w)
    assert flags & PAGE_RANGE
    assert np.isfinite(out).all() and np.isfinite(lse).all()
    ref_out, ref_lse = gh.oracle(b, w, tokens=[2])
    assert_parity(out[2:3], lse[2:3], ref_out, ref_lse, label="intact sequence")


def test_sequence_id_outside_batch(cuda_device):
    w = gh.workload(42, 128, [70, 500, 64])
    b = inputs.materialize(w, cuda_device)
    b.seq_id[1] = 99
    flags, out, lse = _launch(b, w)
    assert flags & SEQ_RANGE
    assert (out[1] == 0).all() and np.isneginf(lse[1]).all()
    ref_out, ref_lse = gh.oracle(b, w, tokens=[0, 2])
    assert_parity(out[[0, 2]], lse[[0, 2]], ref_out, ref_lse, label="valid tokens")


def test_length_beyond_page_table(cuda_device):
    # kv_len past the table's capacity is clamped; q_pos keeps every token inside its pages.
    w = gh.workload(43, 128, [100, 200])
    b = inputs.materialize(w, cuda_device)
    b.kv_len[0] = int(b.page_table.shape[1]) * 64 + 1000
    flags, out, lse = _launch(b, w)
    assert flags & TABLE_SHORT
    ref_out, ref_lse = gh.oracle(b, w)
    assert_parity(out, lse, ref_out, ref_lse, label="clamped length")
