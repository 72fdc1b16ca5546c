"""GPU parity of FP8 E4M3 KV rows (SMLA-C-012, docs/TEST-PLAN.md:225) through the C ABI.

Rows are 512 E4M3 codes and four f32 scales (docs/HOST-CONTRACTS.md:122-123), stride 528 or 544;
q is bf16 [T, H, 512]. The kernel dequantizes each visible row to bf16 in shared memory; the
oracle decodes the same bytes exactly in float64 (oracle/fp8.py) and runs the float64 core.
Rows holding no cached position carry NaN codes and NaN scales: an output that read any of them
would not be finite (NaN containment, SMLA-E-009).
"""

import numpy as np
import pytest
import torch

from conftest import assert_parity
import gpu_helpers as gh
from oracle import fp8 as ofp8
from oracle import mla as omla
from tq_mla import _abi, inputs, ops

pytestmark = pytest.mark.gpu

# The north-star tolerances are stated for bf16 rows, which reach the tensor cores exactly. An FP8
# value (4 significant bits) times its f32 tile scale generally is not a bf16 number, so the
# kernel's dequantized operands carry one more rounding, <= 2^-9 relative per value. Each case is
# checked twice: against the oracle on the operands the kernel computes on (e4m3 x scale rounded
# once to bf16, oracle/fp8.py operand_rows) at the north-star tolerances, and against the oracle
# on the exact dequantized values with lse held to FP8_LSE_ABS. With N(0, 1) latents, N(0, 1)
# queries and scale 1/16, the rounding moves a score by about 0.0625 * sqrt(512 / 3) * 2^-9
# ~ 1.6e-3 (one standard deviation); a query that sees one key has lse equal to that key's score,
# and over ~10^5 (token, head) pairs the largest deviation reaches 6-7 standard deviations.
FP8_LSE_ABS = 2e-2


def _workload(seed, heads, lens, per_seq=1):
    w = gh.workload(seed, heads, lens, per_seq=per_seq, width=512, scale=0.0625)
    w.extra["kv_format"] = "fp8_e4m3"
    w.extra["kv_row_bytes"] = inputs.FP8_ROW_PAYLOAD
    return w


def _run(w, device, row_stride, prefill=False, mutate=None):
    b = inputs.materialize_fp8(w, device, row_stride=row_stride)
    if mutate is not None:
        mutate(b)
    out = torch.empty((w.tokens, w.heads, 512), dtype=torch.bfloat16, device=device)
    lse = torch.empty((w.tokens, w.heads), dtype=torch.float32, device=device)
    launch = ops.MlaLaunch(b.q, b.kv, b.page_table, b.seq_id, b.q_pos, b.kv_len, out, lse,
                           scale=w.scale, query_counts=b.query_counts, prefill=prefill,
                           kv_format=_abi.KV_FP8_E4M3)
    launch()
    torch.cuda.synchronize()
    q = b.q.float().double().cpu().numpy()
    raw = b.kv.reshape(-1, row_stride).cpu().numpy()
    refs = []
    for rows in (ofp8.dequant_rows(raw), ofp8.operand_rows(raw)):
        refs.append(omla.paged_attention(q, rows, w.extra["page_table"], w.seq_id(), w.q_pos(),
                                         w.kv_len, scale=w.scale, value_dim=512))
    return launch, out.float().double().cpu().numpy(), lse.double().cpu().numpy(), refs


def _check(out, lse, refs, label):
    (exact_out, exact_lse), (op_out, op_lse) = refs
    assert_parity(out, lse, op_out, op_lse, label=f"{label} (bf16 operands)")
    assert_parity(out, lse, exact_out, exact_lse, label=f"{label} (exact values)",
                  lse_abs=FP8_LSE_ABS)


@pytest.mark.parametrize("heads,lens,stride", [
    (128, [1, 63, 64, 65, 129, 700, 3000], 544),
    (16, [17, 64, 200, 1000], 528),
])
def test_fp8_decode_matches_oracle(cuda_device, heads, lens, stride):
    w = _workload(71, heads, lens)
    launch, out, lse, refs = _run(w, cuda_device, stride)
    assert launch.device_error() == 0
    assert np.isfinite(out).all() and np.isfinite(lse).all()
    _check(out, lse, refs, f"fp8 decode H={heads} stride={stride}")


@pytest.mark.parametrize("lens,per_seq", [
    ([300, 150, 64], [100, 30, 64]),
    # segments of 5, 4 and 3 pages followed by another segment on the same CTA pair
    ([300, 260, 190, 700], [100, 60, 20, 8]),
])
def test_fp8_causal_prefill_chunks(cuda_device, lens, per_seq):
    w = _workload(72, 128, lens, per_seq=per_seq)
    launch, out, lse, refs = _run(w, cuda_device, 544, prefill=True)
    assert launch.device_error() == 0
    assert np.isfinite(out).all()
    _check(out, lse, refs, f"fp8 prefill {lens}")


def _pool_row(w, seq, pos):
    return int(w.extra["page_table"][seq][pos // 64]) * 64 + pos % 64


def test_fp8_large_scales_and_nan_codes(cuda_device):
    """Tiles the kernel dequantizes through the conversion instructions instead of exponent
    placement: scales of 2^8 and more (subnormal codes keep the values moderate), next to a
    tile with scale 255 on the fast path, and a NaN code in
    a visible row, which makes that token's output and lse NaN (the oracle's too) and leaves the
    other tokens exact."""
    w = _workload(73, 16, [200, 300, 90])
    big_rows = [_pool_row(w, 1, p) for p in (3, 64, 150, 299)]
    nan_row = _pool_row(w, 0, 17)

    def mutate(b):
        flat = b.kv.view(-1, b.kv.shape[-1])
        gen = torch.Generator(device=flat.device)
        gen.manual_seed(5)
        for r in big_rows:
            # codes 0, 1, 2 are 0, 2^-9, 2^-8: times the scales below, values of at most 4
            small = torch.randint(0, 3, (512,), generator=gen, device=flat.device,
                                  dtype=torch.int32).to(torch.uint8)
            sign = (torch.randint(0, 2, (512,), generator=gen, device=flat.device,
                                  dtype=torch.int32) * 0x80).to(torch.uint8)
            flat[r, :512] = small | sign
            sc = torch.tensor([256.0, 300.0, 1024.0, 255.0], device=flat.device)
            flat[r, 512:528] = sc.view(torch.uint8)
        flat[nan_row, 40] = 0x7F

    launch, out, lse, refs = _run(w, cuda_device, 544, mutate=mutate)
    assert launch.device_error() == 0
    assert np.isnan(out[0]).all() and np.isnan(lse[0]).all()
    assert np.isnan(refs[0][0][0]).all()
    keep = [1, 2]
    sub = [(o[keep], l[keep]) for o, l in refs]
    _check(out[keep], lse[keep], sub, "fp8 large scales")
