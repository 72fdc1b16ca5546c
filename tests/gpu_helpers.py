"""Helpers for GPU parity tests: build a seeded paged batch, run the kernel, run the oracle."""

import numpy as np
import torch

from oracle import generate as ogen
from oracle import mla as omla
from tq_mla import inputs, ops


def workload(seed, heads, lens, per_seq=1, width=576, pool_pages=None, prefix=None, scale=None):
    lens = np.asarray(lens, dtype=np.int64)
    q_per = np.full(len(lens), per_seq, dtype=np.int64) if np.isscalar(per_seq) else \
        np.asarray(per_seq, dtype=np.int64)
    if prefix is None:
        prefix = lens - q_per
    if scale is None:
        scale = ops.default_scale(width)
    w = inputs.Workload(f"case_s{seed}", seed, heads, width, lens, q_per,
                        np.asarray(prefix, dtype=np.int64), scale)
    return inputs._finish(w, pool_pages)


def run(w, device, *, out_dtype=torch.bfloat16, prefill=False, row_stride=None):
    b = inputs.materialize(w, device, row_stride=row_stride)
    launch = ops.MlaLaunch(
        b.q, b.kv, b.page_table, b.seq_id, b.q_pos, b.kv_len,
        torch.empty((w.tokens, w.heads, 512), dtype=out_dtype, device=device),
        torch.empty((w.tokens, w.heads), dtype=torch.float32, device=device),
        scale=w.scale, query_counts=b.query_counts, prefill=prefill)
    out, lse = launch()
    torch.cuda.synchronize()
    return b, launch, out, lse


def host_inputs(b, w, row_stride=None):
    """Float64 copies of what the kernel read: q [T,H,D] and pool rows [P*64, D]."""
    q = b.q.float().double().cpu().numpy()
    kv = b.kv
    if kv.dtype == torch.uint8:
        kv = kv[:, :, : w.width * 2].contiguous().view(torch.bfloat16)
    rows = kv.reshape(-1, w.width).float().double().cpu().numpy()
    return q, rows


def oracle(b, w, tokens=None, row_stride=None):
    q, rows = host_inputs(b, w, row_stride)
    return omla.paged_attention(
        q, rows, w.extra["page_table"], w.seq_id(), w.q_pos(), w.kv_len,
        scale=w.scale, value_dim=512, tokens=tokens)


def oracle_inputs_match(b, w):
    """The device generator reproduces the oracle generator bit for bit (q and pool rows)."""
    q_bits = b.q.view(torch.int16).cpu().numpy().view(np.uint16)
    ref_q = np.concatenate([
        ogen.normal_bf16(w.seed, ogen.STREAM_Q, int(w.token_global[s]) * w.heads * w.width,
                         int(w.q_per_seq[s]) * w.heads * w.width)
        for s in range(w.sequences)]).reshape(q_bits.shape)
    kv = b.kv if b.kv.dtype != torch.uint8 else b.kv[:, :, : w.width * 2].contiguous().view(
        torch.bfloat16)
    pool_bits = kv.reshape(-1, w.width).view(torch.int16).cpu().numpy().view(np.uint16)
    ref_pool = ogen.kv_pool(w.seed, w.kv_len, w.extra["page_table"], w.pool_pages, w.width)
    return np.array_equal(q_bits, ref_q), np.array_equal(pool_bits, ref_pool)


def oracle_tokens(b, w, tokens):
    """Oracle ``(out, lse)`` for the selected query ``tokens`` from the device inputs the kernel
    read: each sequence's cached rows are gathered on the device through its page table once,
    widened to float64 on the host, and the token sees its first ``min(kv_len, q_pos + 1)``."""
    table = w.extra["page_table"]
    seq, qpos = w.seq_id(), w.q_pos()
    dev = b.q.device
    order = sorted(int(t) for t in tokens)
    rows_of, cur = None, None
    out = np.zeros((len(order), w.heads, 512))
    lse = np.full((len(order), w.heads), -np.inf)
    for i, t in enumerate(order):
        s = int(seq[t])
        if s != cur:
            n_all = int(w.kv_len[s])
            pages = torch.from_numpy(table[s, : (n_all + 63) // 64].astype(np.int64)).to(dev)
            rows_of = b.kv[pages].reshape(-1, b.kv.shape[-1])[:n_all].double().cpu().numpy()
            cur = s
        n = max(0, min(int(w.kv_len[s]), int(qpos[t]) + 1))
        q = b.q[t].double().cpu().numpy()
        out[i], lse[i] = omla.identity_core(q, rows_of[:n], w.scale, 512)
    return order, out, lse
