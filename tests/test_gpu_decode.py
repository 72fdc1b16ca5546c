"""GPU parity of the paged MLA kernel (tcgen05 path, via the C ABI) against the oracle.

Cases follow the reference's SMLA checklist (docs/TEST-PLAN.md:211-250) where it applies to
dense paged attention: page-edge lengths (C-003, E-003, E-008), shuffled pages (C-005), lse
(C-006), split-KV merge (C-007, E-017), multi-token causal decode (C-004, C-010), NaN
containment in unused slots (E-009), empty sequence inside a batch (E-001, E-008),
determinism (E-013).
"""

import numpy as np
import pytest
import torch

from conftest import GOLDEN, assert_parity
import gpu_helpers as gh
from oracle import schedule as osched
from tq_mla import _abi, ops

pytestmark = pytest.mark.gpu


def _np(t):
    return t.float().double().cpu().numpy()


@pytest.mark.parametrize("name", ["cfg1_decode_h16", "mtp_h32", "nope512_h32"])
def test_golden_cases_from_reference(cuda_device, name):
    g = np.load(GOLDEN / "paged_cases.npz")
    seed, heads, per_seq, width, pool_pages = (int(x) for x in g[f"{name}__meta"])
    w = gh.workload(seed, heads, g[f"{name}__kv_len"], per_seq=per_seq, width=width,
                    pool_pages=pool_pages, scale=float(g[f"{name}__scale"]))
    np.testing.assert_array_equal(w.extra["page_table"], g[f"{name}__page_table"])
    b, launch, out, lse = gh.run(w, cuda_device)
    q_ok, pool_ok = gh.oracle_inputs_match(b, w)
    assert q_ok and pool_ok, "device generator differs from the oracle generator"
    assert launch.device_error() == 0
    assert_parity(_np(out), _np(lse), g[f"{name}__out"], g[f"{name}__lse"], label=name)


@pytest.mark.parametrize("heads", [16, 32, 64, 128])
def test_page_edges_and_heads(cuda_device, heads):
    lens = [1, 2, 63, 64, 65, 127, 128, 129, 200, 1000]
    w = gh.workload(11 + heads, heads, lens)
    b, launch, out, lse = gh.run(w, cuda_device)
    ref_out, ref_lse = gh.oracle(b, w)
    assert launch.device_error() == 0
    assert_parity(_np(out), _np(lse), ref_out, ref_lse, label=f"H={heads}")


def test_multi_token_causal_and_empty_sequence(cuda_device):
    # Two and four query tokens per sequence (C-004); a kv_len = 0 sequence in the batch (E-008).
    lens = [70, 0, 300, 64, 5]
    per = [2, 1, 4, 3, 2]
    prefix = [68, -1, 296, 61, 3]
    w = gh.workload(7, 128, lens, per_seq=per, prefix=prefix)
    b, launch, out, lse = gh.run(w, cuda_device)
    ref_out, ref_lse = gh.oracle(b, w)
    assert_parity(_np(out), _np(lse), ref_out, ref_lse, label="mtp")
    empty = np.flatnonzero(w.visible() == 0)
    assert len(empty) == 1
    assert torch.isneginf(lse[empty[0]]).all()
    assert (out[empty[0]] == 0).all()


def test_long_sequence_split_across_pairs(cuda_device):
    # One long sequence is split over every CTA pair and merged by the combine kernel.
    w = gh.workload(21, 128, [65536 + 17])
    b, launch, out, lse = gh.run(w, cuda_device)
    ref_out, ref_lse = gh.oracle(b, w)
    assert_parity(_np(out), _np(lse), ref_out, ref_lse, label="split")
    layout = ops.workspace_layout(launch.params)
    hdr = launch.workspace[layout.header: layout.header + 64].view(torch.int32).cpu().numpy()
    assert hdr[3] == 1  # one combined token


def test_metadata_matches_schedule_oracle(cuda_device):
    lens = [4096, 1, 0, 8191, 64, 65, 12000, 300]
    w = gh.workload(3, 64, lens, per_seq=[1, 1, 1, 2, 1, 1, 1, 3],
                    prefix=[4095, 0, 0, 8189, 63, 64, 11999, 297])
    b, launch, out, lse = gh.run(w, cuda_device)
    layout = ops.workspace_layout(launch.params)
    ws = launch.workspace.cpu()

    def arr(off, n):
        return ws[off: off + 4 * n].view(torch.int32).numpy()

    t = w.tokens
    meta = osched.partition(w.visible(), layout.pairs)
    hdr = arr(layout.header, 16)
    assert (hdr[0], hdr[1], hdr[2]) == (0, meta["total"], meta["quota"])
    assert hdr[3] == len(meta["combine_units"]) and hdr[4] == len(meta["empty_units"])
    np.testing.assert_array_equal(arr(layout.unit_n, t), w.visible())
    for key, off in (("pages", layout.unit_pages), ("gstart", layout.unit_gstart),
                     ("first_cluster", layout.unit_first), ("nsplit", layout.unit_nsplit),
                     ("split_off", layout.unit_split_off)):
        np.testing.assert_array_equal(arr(off, t), meta[key], err_msg=key)
    np.testing.assert_array_equal(arr(layout.pair_begin, layout.pairs), meta["begin_unit"])
    np.testing.assert_array_equal(arr(layout.combine_list, hdr[3]), meta["combine_units"])
    np.testing.assert_array_equal(arr(layout.empty_list, hdr[4]), meta["empty_units"])
    ref_out, ref_lse = gh.oracle(b, w)
    assert_parity(_np(out), _np(lse), ref_out, ref_lse, label="meta")


def test_deterministic_bitwise(cuda_device):
    w = gh.workload(5, 128, [3000, 77, 5000, 129])
    b, launch, out, lse = gh.run(w, cuda_device)
    o1, l1 = out.clone(), lse.clone()
    for _ in range(3):
        launch()
    torch.cuda.synchronize()
    assert torch.equal(o1.view(torch.int16), out.view(torch.int16))
    assert torch.equal(l1.view(torch.int32), lse.view(torch.int32))
