"""CUDA-graph capture and replay of the decode launch (SMLA-E-013/E-018, docs/TEST-PLAN.md:243,248).

The launch grid depends only on the device (docs/TEST-PLAN.md:205-206), so one captured launch is
valid for any lengths that fit the captured buffers. The test captures a decode call once, then
rewrites kv_len and q_pos in place (never longer than the generated sequences, so every visible
row holds data) and replays: each replay matches the oracle for the lengths it saw, and repeated
replays of the same lengths are bitwise identical.
"""

import numpy as np
import pytest
import torch

from conftest import assert_parity
import gpu_helpers as gh
from oracle import mla as omla
from tq_mla import inputs, ops

pytestmark = pytest.mark.gpu


def _np(t):
    return t.float().double().cpu().numpy()


def test_graph_replay_with_new_lengths_is_exact_and_deterministic(cuda_device):
    lens0 = [700, 3000, 64, 1500, 129]
    w = gh.workload(61, 128, lens0)
    b = inputs.materialize(w, cuda_device)
    out = torch.empty((w.tokens, w.heads, 512), dtype=torch.bfloat16, device=cuda_device)
    lse = torch.empty((w.tokens, w.heads), dtype=torch.float32, device=cuda_device)
    launch = ops.MlaLaunch(b.q, b.kv, b.page_table, b.seq_id, b.q_pos, b.kv_len, out, lse,
                           scale=w.scale, query_counts=b.query_counts)
    stream = torch.cuda.Stream(cuda_device)
    with torch.cuda.stream(stream):
        launch(stream)  # first call outside the capture: one-time library set-up
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        launch(stream)
    q, rows = gh.host_inputs(b, w)
    for lens in (lens0, [1, 2047, 63, 700, 65], [300, 64, 1, 1499, 128]):
        kv_len = np.asarray(lens, dtype=np.int64)
        q_pos = kv_len - 1
        b.kv_len.copy_(torch.as_tensor(kv_len, dtype=torch.int32))
        b.q_pos.copy_(torch.as_tensor(q_pos, dtype=torch.int32))
        torch.cuda.synchronize()
        graph.replay()
        torch.cuda.synchronize()
        assert launch.device_error() == 0
        ref_out, ref_lse = omla.paged_attention(q, rows, w.extra["page_table"], w.seq_id(), q_pos,
                                                kv_len, scale=w.scale, value_dim=512)
        assert_parity(_np(out), _np(lse), ref_out, ref_lse, label=f"replay {lens}")
        first_out, first_lse = out.clone(), lse.clone()
        for rep in range(100):  # bitwise determinism over 100 runs (docs/TEST-PLAN.md:243)
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, first_out) and torch.equal(lse, first_lse), (lens, rep)
