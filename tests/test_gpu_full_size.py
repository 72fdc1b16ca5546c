"""GPU parity at the benchmark configurations' real sizes (C ABI against the oracle).

The launch metadata (split-KV partition, split counts per token, combine fan-in) depends on the
batch shape, so each configuration is checked as it is timed:
  - decode: the whole 64-sequence batch, 128 heads, lengths U[4096, 8192] (every token);
  - prefill: full 2048-token chunks after prefixes of 0 and 6144 positions (first, middle, last
    and 64 random query tokens of each chunk);
  - long context: the 4 x 131072-position batch on one GPU, and the same batch split over 8
    page ranges (one per device of an 8-GPU job, run in turn here) merged by tq_mla_combine;
  - multi-token decode: the 512 x 2-token log-normal batch (lengths clipped to [256, 65536]),
    checked on every clipped sequence plus a spread of others, both query tokens each.
Tolerances are the north-star ones (out max-abs 2e-2, relative L2 1e-2; lse 1e-3).
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


def _launch(w, dev, *, prefill=False, out_dtype=torch.bfloat16):
    b = inputs.materialize(w, dev)
    launch = ops.MlaLaunch(
        b.q, b.kv, b.page_table, b.seq_id, b.q_pos, b.kv_len,
        torch.empty((w.tokens, w.heads, 512), dtype=out_dtype, device=dev),
        torch.empty((w.tokens, w.heads), dtype=torch.float32, device=dev),
        scale=w.scale, query_counts=b.query_counts, prefill=prefill)
    out, lse = launch()
    torch.cuda.synchronize()
    assert launch.device_error() == 0
    return b, launch, out, lse


def _check(b, w, out, lse, tokens, label):
    order, ref_out, ref_lse = gh.oracle_tokens(b, w, tokens)
    assert_parity(_np(out[order]), _np(lse[order]), ref_out, ref_lse, label=label)


def test_decode_whole_batch(cuda_device):
    w = inputs.config("decode")
    assert w.sequences == 64 and w.heads == 128 and w.kv_len.min() >= 4096
    b, launch, out, lse = _launch(w, cuda_device)
    layout = ops.workspace_layout(launch.params)
    header = launch.workspace[: 64].view(torch.int32).cpu().numpy()
    assert header[3] > 0, "the timed decode batch splits tokens across CTA pairs"
    _check(b, w, out, lse, range(w.tokens), "decode b64")
    assert layout.pairs > 0


def test_prefill_full_chunks(cuda_device):
    pre = np.array([0, 6144], dtype=np.int64)
    w = inputs.Workload("prefill_full_chunks", 2, 128, 576, pre + 2048, np.full(2, 2048), pre,
                        ops.default_scale(576))
    w = inputs._finish(w)
    b, launch, out, lse = _launch(w, cuda_device, prefill=True)
    rng = np.random.default_rng(5)
    picks = []
    for s in range(2):
        base = 2048 * s
        local = np.concatenate([np.arange(64), 992 + np.arange(64), 1984 + np.arange(64),
                                rng.choice(2048, 64, replace=False)])
        picks.extend(base + np.unique(local))
    _check(b, w, out, lse, picks, "prefill 2x2048")


def test_long_context_batch_and_eight_way_split(cuda_device):
    w = inputs.config("longctx")
    assert (w.kv_len == 131072).all()
    b, _, out, lse = _launch(w, cuda_device)
    order, ref_out, ref_lse = gh.oracle_tokens(b, w, range(w.tokens))
    assert_parity(_np(out[order]), _np(lse[order]), ref_out, ref_lse, label="longctx")
    del b
    torch.cuda.empty_cache()
    parts_out, parts_lse = [], []
    for r in range(8):
        sub = tdist.context_split(w, 8, r)
        _, _, po, pl = _launch(sub, cuda_device, out_dtype=torch.float32)
        parts_out.append(po)
        parts_lse.append(pl)
    m_out, m_lse = ops.combine_parts(torch.stack(parts_out), torch.stack(parts_lse))
    torch.cuda.synchronize()
    assert_parity(_np(m_out), _np(m_lse), ref_out, ref_lse, label="longctx split x8")


def test_multi_token_lognormal_batch(cuda_device):
    w = inputs.config("mtp")
    assert w.sequences == 512 and (w.q_per_seq == 2).all()
    clipped = np.flatnonzero(w.kv_len == 65536)
    assert len(clipped) >= 1 and w.kv_len.min() >= 256
    b, _, out, lse = _launch(w, cuda_device)
    spread = np.unique(np.linspace(0, w.sequences - 1, 24).astype(int))
    shortest = np.argsort(w.kv_len)[:4]
    seqs = np.unique(np.concatenate([clipped, spread, shortest]))
    starts = np.concatenate([[0], np.cumsum(w.q_per_seq)[:-1]])
    tokens = np.concatenate([starts[s] + np.arange(2) for s in seqs])
    _check(b, w, out, lse, tokens, "mtp 512x2")
