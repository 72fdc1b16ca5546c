"""The no-allocation decode entry point against the regular one (GPU).

``tq_mla_decode_no_alloc`` serves callers that cannot allocate device memory when they launch
(an engine that gives all GPU memory to its own pool at start-up, or code where cudaMalloc is
not allowed): it runs the same scheduler, attention and combine kernels as ``tq_mla_decode`` but
on a fixed workspace array inside the library. This test calls it through the C ABI twice in a
row, on two different batches, so the second call runs over the first call's leftover workspace,
and checks each result against ``tq_mla_decode`` with a caller-allocated workspace, within the
parity tolerances of the other GPU tests, with the device error flags of each call read back
through tq_mla_no_alloc_read_device_error. Sparse top-k plans (bf16 and FP8 rows), which keep
their compacted entries after the partials in the same array, are checked the same way. It also
checks that dense and sparse plans too large for the fixed array are refused with
TQ_ERR_WORKSPACE. The file name makes pytest collect it last.
"""

import ctypes

import numpy as np
import pytest
import torch

from conftest import assert_parity
import gpu_helpers as gh
from tq_mla import _abi, inputs, ops

pytestmark = pytest.mark.gpu


def _np(t):
    return t.float().double().cpu().numpy()


def _no_alloc_decode(w, device):
    """Run one batch through tq_mla_decode_no_alloc; returns (batch, out, lse), float64 results."""
    b = inputs.materialize(w, device)
    out = torch.full((w.tokens, w.heads, 512), float("nan"), dtype=torch.bfloat16, device=device)
    lse = torch.full((w.tokens, w.heads), float("nan"), dtype=torch.float32, device=device)
    spec = ops.make_spec(b.q, b.kv, b.page_table, b.seq_id, b.q_pos, b.kv_len, out, lse,
                         scale=w.scale)
    params = ops.validate(spec, b.query_counts)
    err = _abi.TqContractError()
    stream = torch.cuda.current_stream(device)
    status = _abi.lib.tq_mla_decode_no_alloc(ctypes.byref(params),
                                             ctypes.c_void_p(stream.cuda_stream),
                                             ctypes.byref(err))
    _abi.raise_for(status, err)
    torch.cuda.synchronize(device)
    assert _no_alloc_flags(stream) == 0
    return b, _np(out), _np(lse)


def _no_alloc_flags(stream):
    flags = ctypes.c_int32(-1)
    _abi.raise_for(_abi.lib.tq_mla_no_alloc_read_device_error(ctypes.c_void_p(stream.cuda_stream),
                                                              ctypes.byref(flags)))
    return flags.value


def _sparse_plan(w, b, k, rng, device, fmt=None, tokens=None):
    """A sparse top-k plan over batch ``b``: per token up to ``k`` random valid positions, then
    -1 entries. Returns (params, out, lse, launch with a caller workspace)."""
    seq, q_pos = w.seq_id(), w.q_pos()
    idx = np.full((w.tokens, k), -1, np.int32)
    for t in range(w.tokens):
        vis = int(min(w.kv_len[seq[t]], q_pos[t] + 1))
        n = min(vis, k)
        idx[t, :n] = rng.choice(vis, size=n, replace=False)
    d_idx = torch.from_numpy(idx).to(device)
    d_klen = torch.full((w.tokens,), k, dtype=torch.int32, device=device)
    out = torch.full((w.tokens, w.heads, 512), float("nan"), dtype=torch.bfloat16, device=device)
    lse = torch.full((w.tokens, w.heads), float("nan"), dtype=torch.float32, device=device)
    launch = ops.MlaLaunch(b.q, b.kv, b.page_table, b.seq_id, b.q_pos, b.kv_len, out, lse,
                           scale=0.0625, query_counts=b.query_counts, kv_format=fmt, idx=d_idx,
                           k_len=d_klen)
    return launch, out, lse


def test_no_alloc_matches_regular_entry_point_twice(cuda_device):
    # Lengths cross page edges and, with the CTA pairs sharing few pages, most tokens are split
    # across pairs, so the partial-result slots of the workspace are used and reused.
    first = gh.workload(101, 128, [17, 64, 200, 1000, 4097, 65, 1, 129])
    second = gh.workload(202, 128, [3000, 7, 64, 513, 0, 2048], per_seq=[1, 1, 2, 1, 1, 3],
                         prefix=[2999, 6, 62, 512, -1, 2045])
    for label, w in (("first call", first), ("second call", second)):
        _, out, lse = _no_alloc_decode(w, cuda_device)
        _, launch, ref_out, ref_lse = gh.run(w, cuda_device)
        assert launch.device_error() == 0
        assert_parity(out, lse, _np(ref_out), _np(ref_lse), label=label)


def test_no_alloc_rejects_plans_beyond_the_fixed_workspace(cuda_device):
    # A plan whose workspace exceeds the fixed 42 MiB array is refused before any launch. On a
    # B200 the split partials take about 39 MB and each query token 32 bytes, so 200 000 tokens
    # (50 000 sequences x 4 queries, the decode maximum, 16 heads) are over the limit.
    limit = 42 << 20
    seqs, per = 50_000, 4
    tokens = seqs * per
    dev = cuda_device
    w = gh.workload(5, 16, [1])
    kv = inputs.materialize(w, dev).kv
    q = torch.empty((tokens, 16, 576), dtype=torch.bfloat16, device=dev)
    page_table = torch.zeros((seqs, 1), dtype=torch.int32, device=dev)
    seq_id = torch.arange(seqs, dtype=torch.int32, device=dev).repeat_interleave(per)
    q_pos = torch.zeros(tokens, dtype=torch.int32, device=dev)
    kv_len = torch.ones(seqs, dtype=torch.int32, device=dev)
    out = torch.empty((tokens, 16, 512), dtype=torch.bfloat16, device=dev)
    lse = torch.empty((tokens, 16), dtype=torch.float32, device=dev)
    spec = ops.make_spec(q, kv, page_table, seq_id, q_pos, kv_len, out, lse, scale=w.scale)
    params = ops.validate(spec, [per] * seqs)
    assert ops.workspace_bytes(params, dev.index) > limit
    err = _abi.TqContractError()
    status = _abi.lib.tq_mla_decode_no_alloc(ctypes.byref(params), None, ctypes.byref(err))
    assert status == 102  # TQ_ERR_WORKSPACE
    assert err.field == b"no_alloc_workspace"


@pytest.mark.parametrize("fmt", ["bf16", "fp8"])
def test_no_alloc_sparse_plans_match_regular_entry_point(cuda_device, fmt):
    w = gh.workload(303, 32, [1, 63, 64, 65, 2047, 4096], per_seq=[1, 1, 2, 1, 3, 2], width=512,
                    scale=0.0625)
    if fmt == "fp8":
        b = inputs.materialize_fp8(w, cuda_device, row_stride=544)
        kv_fmt = _abi.KV_FP8_E4M3
    else:
        b = inputs.materialize(w, cuda_device)
        kv_fmt = None
    launch, out, lse = _sparse_plan(w, b, 512, np.random.default_rng(9), cuda_device, kv_fmt)
    stream = torch.cuda.current_stream(cuda_device)
    for call in range(2):
        out.fill_(float("nan"))
        err = _abi.TqContractError()
        _abi.raise_for(_abi.lib.tq_mla_decode_no_alloc(ctypes.byref(launch.params),
                                                       ctypes.c_void_p(stream.cuda_stream),
                                                       ctypes.byref(err)), err)
        torch.cuda.synchronize(cuda_device)
        assert _no_alloc_flags(stream) == 0
        got_out, got_lse = _np(out), _np(lse)
        ref_out, ref_lse = launch()
        torch.cuda.synchronize(cuda_device)
        assert launch.device_error() == 0
        assert_parity(got_out, got_lse, _np(ref_out), _np(ref_lse), label=f"sparse {fmt} {call}")


def test_no_alloc_rejects_sparse_plans_beyond_the_fixed_workspace(cuda_device):
    # 2051 entries per token cost 8 208 bytes of the array each: 1 024 tokens are over the limit.
    limit = 42 << 20
    seqs, k = 1024, 2051
    dev = cuda_device
    w = gh.workload(6, 32, [1], width=512, scale=0.0625)
    kv = inputs.materialize(w, dev).kv
    q = torch.empty((seqs, 32, 512), dtype=torch.bfloat16, device=dev)
    page_table = torch.zeros((seqs, 1), dtype=torch.int32, device=dev)
    seq_id = torch.arange(seqs, dtype=torch.int32, device=dev)
    q_pos = torch.zeros(seqs, dtype=torch.int32, device=dev)
    kv_len = torch.ones(seqs, dtype=torch.int32, device=dev)
    out = torch.empty((seqs, 32, 512), dtype=torch.bfloat16, device=dev)
    lse = torch.empty((seqs, 32), dtype=torch.float32, device=dev)
    idx = torch.full((seqs, k), -1, dtype=torch.int32, device=dev)
    k_len = torch.zeros(seqs, dtype=torch.int32, device=dev)
    spec = ops.make_spec(q, kv, page_table, seq_id, q_pos, kv_len, out, lse, scale=0.0625)
    params = ops.validate(spec, [1] * seqs, idx=ops.spec_of(idx), k_len=ops.spec_of(k_len))
    assert ops.workspace_bytes(params, dev.index) > limit
    err = _abi.TqContractError()
    status = _abi.lib.tq_mla_decode_no_alloc(ctypes.byref(params), None, ctypes.byref(err))
    assert status == 102 and err.field == b"no_alloc_workspace"
