"""GPU parity of the launch paths beyond single-batch bf16 decode (C ABI against the oracle).

  - causal chunked prefill through ``tq_mla_prefill`` (many query tokens per sequence over a
    cached prefix; the SMLA-PF plan, docs/TEST-PLAN.md:195,410-413);
  - f32 output (the per-device partial of a cross-device split);
  - KV rows with a padded stride (contracts.rs:359-371 allow stride >= payload, % 16 == 0);
  - a cross-device context split run as two partial launches and merged by ``tq_mla_combine``
    (the long-context row of the multi-GPU plan, merged by log-sum-exp as mla_attention.py:152-169).
"""

import numpy as np
import pytest
import torch

from conftest import assert_parity
import gpu_helpers as gh
from tq_mla import dist as tdist
from tq_mla import inputs, ops

pytestmark = pytest.mark.gpu


def _np(t):
    return t.float().double().cpu().numpy()


def test_prefill_causal_chunks(cuda_device):
    # Chunks of new tokens after a cached prefix: token t sees positions [0, q_pos[t]].
    lens = [150, 300, 64, 1]
    per = [30, 100, 64, 1]
    w = gh.workload(31, 128, lens, per_seq=per)
    b, launch, out, lse = gh.run(w, cuda_device, prefill=True)
    ref_out, ref_lse = gh.oracle(b, w)
    assert launch.device_error() == 0
    assert_parity(_np(out), _np(lse), ref_out, ref_lse, label="prefill")


def test_f32_output(cuda_device):
    w = gh.workload(32, 128, [5, 64, 65, 700, 2500])
    b, launch, out, lse = gh.run(w, cuda_device, out_dtype=torch.float32)
    assert out.dtype == torch.float32
    ref_out, ref_lse = gh.oracle(b, w)
    assert launch.device_error() == 0
    assert_parity(_np(out), _np(lse), ref_out, ref_lse, label="f32 out")


def test_padded_kv_row_stride(cuda_device):
    w = gh.workload(33, 64, [1, 63, 64, 129, 1000])
    b, launch, out, lse = gh.run(w, cuda_device, row_stride=1280)
    ref_out, ref_lse = gh.oracle(b, w, row_stride=1280)
    assert launch.device_error() == 0
    assert_parity(_np(out), _np(lse), ref_out, ref_lse, label="padded rows")


def test_context_split_merged_on_device(cuda_device):
    # Each "device" computes f32 partials over its page range; tq_mla_combine merges them.
    w = gh.workload(34, 128, [3000, 129, 64, 640])
    full = inputs.materialize(w, cuda_device)
    ref_out, ref_lse = gh.oracle(full, w)
    parts_out, parts_lse = [], []
    for r in range(2):
        sub = tdist.context_split(w, 2, r)
        _, launch, out, lse = gh.run(sub, cuda_device, out_dtype=torch.float32)
        assert launch.device_error() == 0
        parts_out.append(out)
        parts_lse.append(lse)
    out, lse = ops.combine_parts(torch.stack(parts_out), torch.stack(parts_lse))
    torch.cuda.synchronize()
    assert_parity(_np(out), _np(lse), ref_out, ref_lse, label="context split")
    # The 64-row sequence has a single page, so exactly one part saw no key: lse -inf there.
    empty = [bool(np.isneginf(_np(l)[2]).all()) for l in parts_lse]
    assert sorted(empty) == [False, True]
