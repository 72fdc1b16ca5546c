"""GPU: sparse top-k decode plans through the C ABI (docs/TEST-PLAN.md:174-248, SMLA-C/E).

Token t attends to the rows of its valid index entries: j < k_len[t], 0 <= idx <= q_pos[t] and
idx < kv_len (docs/TEST-PLAN.md:199). The oracle (oracle/mla.py sparse_attention) gathers the same
rows in float64. Pools come from the seeded generators with permuted pages, and rows that hold no
cached position are NaN-poisoned, so an invalid entry that was read would show as NaN.
"""

import dataclasses

import numpy as np
import pytest
import torch

from conftest import assert_parity
import gpu_helpers as gh
from oracle import fp8 as ofp8
from oracle import mla as omla
from tq_mla import _abi, inputs, ops

pytestmark = pytest.mark.gpu

SCALE = 0.0625  # 256 ** -0.5, the contract's fixed scale
I32_MAX, I32_MIN = 2 ** 31 - 1, -2 ** 31


def _np(t):
    return t.float().double().cpu().numpy()


def _indices(rng, w, k, q_pos, junk=True):
    """Per token: up to k unique valid positions in random order, padded with invalid entries
    (-1, > q_pos, >= kv_len, extremes) and stale values after k_len."""
    seq = w.seq_id()
    idx = np.full((w.tokens, k), -1, np.int32)
    k_len = np.zeros(w.tokens, np.int32)
    for t in range(w.tokens):
        vis = int(min(w.kv_len[seq[t]], q_pos[t] + 1))
        n = min(vis, k - (8 if junk else 0))
        sel = rng.choice(vis, size=n, replace=False).astype(np.int32) if n > 0 else np.zeros(0, np.int32)
        bad = np.array([-1, int(q_pos[t]) + 1, int(w.kv_len[seq[t]]), I32_MAX, -2, I32_MIN, -1,
                        int(w.kv_len[seq[t]]) + 64], np.int64).clip(I32_MIN, I32_MAX).astype(np.int32)
        row = np.concatenate([sel, bad[: k - n]]) if junk else sel
        rng.shuffle(row)
        idx[t, : len(row)] = row
        k_len[t] = len(row)
        if k_len[t] < k:  # stale in-range values after k_len are ignored (SMLA-E-019)
            idx[t, k_len[t]:] = rng.integers(0, max(1, vis), size=k - k_len[t])
    return idx, k_len


def _launch(b, w, idx, k_len, device, fmt=None, idx_pad=0):
    d_idx = torch.from_numpy(idx).to(device)
    if idx_pad:
        wide = torch.full((idx.shape[0], idx.shape[1] + idx_pad), 7, dtype=torch.int32,
                          device=device)
        wide[:, : idx.shape[1]] = d_idx
        d_idx = wide[:, : idx.shape[1]]
    d_klen = torch.from_numpy(k_len).to(device)
    out = torch.empty((w.tokens, w.heads, 512), dtype=torch.bfloat16, device=device)
    lse = torch.empty((w.tokens, w.heads), dtype=torch.float32, device=device)
    launch = ops.MlaLaunch(b.q, b.kv, b.page_table, b.seq_id, b.q_pos, b.kv_len, out, lse,
                           scale=SCALE, query_counts=b.query_counts, kv_format=fmt, idx=d_idx,
                           k_len=d_klen)
    return launch, out, lse, d_idx, d_klen


@pytest.mark.parametrize("heads", [32, 64, 128])
def test_sparse_bf16_matches_oracle(cuda_device, heads):
    lens = [1, 63, 64, 65, 2047, 4096, 32768]
    w = gh.workload(81 + heads, heads, lens, per_seq=[1, 1, 2, 1, 3, 4, 1], width=512, scale=SCALE)
    b = inputs.materialize(w, cuda_device)
    rng = np.random.default_rng(heads)
    idx, k_len = _indices(rng, w, 2048, w.q_pos())
    launch, out, lse, _, _ = _launch(b, w, idx, k_len, cuda_device, idx_pad=13)
    launch()
    torch.cuda.synchronize()
    assert launch.device_error() == 0
    q, rows = gh.host_inputs(b, w)
    ref_out, ref_lse = omla.sparse_attention(q, rows, w.extra["page_table"], w.seq_id(), w.q_pos(),
                                             w.kv_len, idx, k_len, scale=SCALE)
    assert np.isfinite(_np(out)).all()
    assert_parity(_np(out), lse.double().cpu().numpy(), ref_out, ref_lse,
                  label=f"sparse bf16 H={heads}")


@pytest.mark.parametrize("stride", [528, 544])
def test_sparse_fp8_matches_oracle(cuda_device, stride):
    from test_gpu_fp8 import FP8_LSE_ABS, _workload

    w = _workload(91, 32, [65, 700, 4096, 20000], per_seq=[1, 2, 4, 3])
    b = inputs.materialize_fp8(w, cuda_device, row_stride=stride)
    rng = np.random.default_rng(stride)
    idx, k_len = _indices(rng, w, 2051, w.q_pos())
    launch, out, lse, _, _ = _launch(b, w, idx, k_len, cuda_device, fmt=_abi.KV_FP8_E4M3)
    launch()
    torch.cuda.synchronize()
    assert launch.device_error() == 0
    q = _np(b.q)
    raw = b.kv.reshape(-1, stride).cpu().numpy()
    for rows, lse_abs, label in ((ofp8.operand_rows(raw), None, "bf16 operands"),
                                 (ofp8.dequant_rows(raw), FP8_LSE_ABS, "exact values")):
        ref_out, ref_lse = omla.sparse_attention(q, rows, w.extra["page_table"], w.seq_id(),
                                                 w.q_pos(), w.kv_len, idx, k_len, scale=SCALE)
        kw = {} if lse_abs is None else {"lse_abs": lse_abs}
        assert_parity(_np(out), lse.double().cpu().numpy(), ref_out, ref_lse,
                      label=f"sparse fp8 stride {stride} ({label})", **kw)


def _probe_pool(device, lens, rng):
    """One-hot rows: position i of each sequence holds e_(i % 512) (bf16 1.0), pages permuted."""
    pages_per = [max(1, -(-n // 64)) for n in lens]
    total = sum(pages_per)
    perm = rng.permutation(total).astype(np.int32)
    table = np.full((len(lens), max(pages_per)), -1, np.int32)
    pool = np.zeros((total * 64, 512), np.float32)
    at = 0
    for s, (n, np_) in enumerate(zip(lens, pages_per)):
        table[s, :np_] = perm[at: at + np_]
        at += np_
        for i in range(n):
            pool[table[s, i // 64] * 64 + i % 64, i % 512] = 1.0
    kv = torch.from_numpy(pool).to(torch.bfloat16).reshape(total, 64, 512).to(device)
    return kv, table


def test_exact_index_set_probe(cuda_device):
    """SMLA-C-011 / E-003 / E-004 / E-005 / E-019 / C-010: q = 0, so every valid entry weighs
    1/n; rows are one-hot, so the output's support is exactly the valid set, each value is 1/n
    to bf16 rounding and lse = ln n."""
    rng = np.random.default_rng(5)
    counts = [1, 2, 15, 16, 17, 63, 64, 65, 127, 128, 129, 500, 512]
    lens = [512] * len(counts) + [1, 64, 65, 0]   # kv_len = 1, page edges, an empty sequence
    heads, k = 32, 2051
    s_count = len(lens)
    kv, table = _probe_pool(cuda_device, lens, rng)
    t_count = s_count
    seq_id = np.arange(s_count, dtype=np.int32)
    q_pos = np.array([511] * len(counts) + [0, 63, 64, 0], np.int32)
    kv_len = np.array(lens, np.int32)
    idx = np.full((t_count, k), -1, np.int32)
    k_len = np.zeros(t_count, np.int32)
    want = []
    for t in range(t_count):
        vis = int(min(kv_len[t], q_pos[t] + 1))
        n = counts[t] if t < len(counts) else vis
        sel = rng.choice(vis, size=n, replace=False) if n else np.zeros(0, np.int64)
        # -1 leading, trailing and interleaved; out-of-range values; a causal violation
        junk = [-1, int(q_pos[t]) + 1, int(kv_len[t]), I32_MAX, -2, I32_MIN, -1]
        row = list(junk[:3]) + [int(x) for x in sel[: n // 2]] + [-1] + \
            [int(x) for x in sel[n // 2:]] + junk[3:]
        row = row[:k]
        idx[t, : len(row)] = row
        k_len[t] = len(row)
        idx[t, k_len[t]:] = rng.integers(0, max(1, vis), size=k - k_len[t])  # stale padding
        want.append(np.sort(sel))
    q = torch.zeros((t_count, heads, 512), dtype=torch.bfloat16, device=cuda_device)
    dev = lambda a: torch.from_numpy(a).to(cuda_device)
    out = torch.empty((t_count, heads, 512), dtype=torch.bfloat16, device=cuda_device)
    lse = torch.empty((t_count, heads), dtype=torch.float32, device=cuda_device)
    ops.mla_decode(q, kv, dev(table), dev(seq_id), dev(q_pos), dev(kv_len), scale=SCALE,
                   query_counts=[1] * s_count, out=out, lse=lse, idx=dev(idx), k_len=dev(k_len))
    torch.cuda.synchronize()
    o = _np(out)
    l_ = lse.double().cpu().numpy()
    for t in range(t_count):
        n = len(want[t])
        if n == 0:
            assert (o[t] == 0).all() and np.isneginf(l_[t]).all(), t
            continue
        support = np.flatnonzero(o[t, 0])
        assert np.array_equal(support, want[t] % 512), (t, n)
        expect = float(torch.tensor(1.0 / n, dtype=torch.bfloat16))
        assert (o[t][:, support] == expect).all(), (t, n)
        assert np.abs(l_[t] - np.log(n)).max() <= 2e-6, (t, n, l_[t, 0])


def test_empty_index_rows_give_zeros_and_neg_inf(cuda_device):
    """SMLA-E-001 / E-008: all -1, k_len = 0, and a kv_len = 0 sequence inside the batch."""
    w = gh.workload(7, 64, [300, 0, 129], width=512, scale=SCALE)
    b = inputs.materialize(w, cuda_device)
    idx = np.full((w.tokens, 64), -1, np.int32)
    k_len = np.array([64, 0, 0], np.int32)
    idx[2, :] = np.arange(64)              # valid values, but k_len = 0
    idx[1, :5] = [0, 1, 2, 3, 4]           # the empty sequence: idx >= kv_len
    k_len[1] = 5
    launch, out, lse, _, _ = _launch(b, w, idx, k_len, cuda_device)
    launch()
    torch.cuda.synchronize()
    assert launch.device_error() == 0
    assert (_np(out) == 0).all() and np.isneginf(lse.cpu().numpy()).all()


def test_nan_in_unselected_rows_changes_nothing(cuda_device):
    """SMLA-E-009: NaN in every row no valid entry selects, page 0 row 0 included: the output is
    bitwise equal to the clean run."""
    w = gh.workload(9, 64, [3000, 700, 64], per_seq=[2, 1, 1], width=512, scale=SCALE)
    b = inputs.materialize(w, cuda_device)
    rng = np.random.default_rng(9)
    idx, k_len = _indices(rng, w, 512, w.q_pos())
    launch, out, lse, _, _ = _launch(b, w, idx, k_len, cuda_device)
    launch()
    torch.cuda.synchronize()
    clean_out, clean_lse = out.clone(), lse.clone()
    used = np.zeros(b.kv.shape[0] * 64, bool)
    seq, qp = w.seq_id(), w.q_pos()
    table = w.extra["page_table"]
    for t in range(w.tokens):
        v = omla.sparse_entries(idx[t], k_len[t], qp[t], w.kv_len[seq[t]])
        used[table[seq[t]][v // 64].astype(np.int64) * 64 + v % 64] = True
    flat = b.kv.view(-1, 512)
    flat[torch.from_numpy(~used).to(cuda_device)] = float("nan")
    assert torch.isnan(flat[0]).all() or used[0]
    launch()
    torch.cuda.synchronize()
    assert torch.equal(out, clean_out) and torch.equal(lse, clean_lse)


def test_graph_replay_with_new_indices_is_exact_and_deterministic(cuda_device):
    """SMLA-E-013 / E-018: one captured launch replayed with new idx, k_len, q_pos and kv_len;
    each replay matches the oracle and repeated replays are bitwise identical."""
    lens = [4000, 1500, 2048, 300]
    w = gh.workload(13, 64, lens, per_seq=[2, 1, 1, 1], width=512, scale=SCALE)
    b = inputs.materialize(w, cuda_device)
    rng = np.random.default_rng(13)
    k = 2048
    idx, k_len = _indices(rng, w, k, w.q_pos())
    launch, out, lse, d_idx, d_klen = _launch(b, w, idx, k_len, cuda_device)
    stream = torch.cuda.Stream(cuda_device)
    with torch.cuda.stream(stream):
        launch(stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        launch(stream)
    q, rows = gh.host_inputs(b, w)
    for rep in range(3):
        if rep:
            kv_len = np.minimum(w.kv_len, rng.integers(1, w.kv_len + 1)).astype(np.int32)
            q_pos = np.concatenate([np.full(c, kl - 1) for c, kl in zip(w.q_per_seq, kv_len)])
            q_pos = (q_pos - np.concatenate([np.arange(c)[::-1] for c in w.q_per_seq])).clip(0)
            w2 = dataclasses.replace(w, kv_len=kv_len.astype(np.int64))
            idx, k_len = _indices(rng, w2, k, q_pos)
            b.kv_len.copy_(torch.from_numpy(kv_len))
            b.q_pos.copy_(torch.from_numpy(q_pos.astype(np.int32)))
            d_idx.copy_(torch.from_numpy(idx))
            d_klen.copy_(torch.from_numpy(k_len))
        else:
            kv_len, q_pos = w.kv_len.astype(np.int32), w.q_pos()
        torch.cuda.synchronize()
        graph.replay()
        torch.cuda.synchronize()
        assert launch.device_error() == 0
        ref_out, ref_lse = omla.sparse_attention(q, rows, w.extra["page_table"], w.seq_id(),
                                                 q_pos, kv_len, idx, k_len, scale=SCALE)
        assert_parity(_np(out), lse.double().cpu().numpy(), ref_out, ref_lse,
                      label=f"sparse replay {rep}")
        first = out.clone(), lse.clone()
        for i in range(100):  # bitwise determinism over 100 runs (docs/TEST-PLAN.md:243)
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, first[0]) and torch.equal(lse, first[1]), (rep, i)


@pytest.mark.parametrize("name", ["sparse_h32", "sparse_k2051"])
def test_sparse_golden_cases_from_reference(cuda_device, name):
    """The kernel on the seeded inputs of tests/golden/sparse_cases.npz against the reference's
    mla_attention_core run with each token's valid-position mask."""
    from conftest import GOLDEN

    g = np.load(GOLDEN / "sparse_cases.npz")
    seed, heads, width, pool_pages = (int(x) for x in g[f"{name}__meta"])
    w = gh.workload(seed, heads, g[f"{name}__kv_len"], per_seq=g[f"{name}__per_seq"],
                    width=width, pool_pages=pool_pages, scale=float(g[f"{name}__scale"]))
    np.testing.assert_array_equal(w.extra["page_table"], g[f"{name}__page_table"])
    b = inputs.materialize(w, cuda_device)
    q_ok, pool_ok = gh.oracle_inputs_match(b, w)
    assert q_ok and pool_ok, "device generator differs from the oracle generator"
    np.testing.assert_array_equal(w.q_pos(), g[f"{name}__q_pos"])
    launch, out, lse, _, _ = _launch(b, w, g[f"{name}__idx"], g[f"{name}__k_len"], cuda_device)
    launch()
    torch.cuda.synchronize()
    assert launch.device_error() == 0
    assert_parity(_np(out), lse.double().cpu().numpy(), g[f"{name}__out"], g[f"{name}__lse"],
                  label=name)
