"""GPU parity of the cross-device context split through ``tq_mla_context_merge`` (C ABI, NCCL).

Each rank decodes its page range of every sequence into f32 partials; the library all-gathers
the partials over its own NCCL communicator and merges them by log-sum-exp (decode context
parallelism, docs/ARCHITECTURE.md:240-241,313). Checked against the oracle over the whole
sequences:
  - one GPU: a communicator of one rank (the all-gather is a copy) over an 8-part split run in
    turn, merged part by part through the C entry point and with tq_mla_combine;
  - two GPUs (when the box has them): two ranks in two processes, each with its own GPU.
The peer-memory merge (``tq_peer_merge_*``: partials read over NVLink, no collective on the step)
is checked the same way: one rank over two steps, two ranks over three.
"""

import os
import socket

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


def _partial(w, dev, out=None, lse=None):
    """This rank's f32 partial of workload ``w`` (into ``out`` / ``lse`` when given)."""
    b = inputs.materialize(w, dev)
    launch = ops.MlaLaunch(
        b.q, b.kv, b.page_table, b.seq_id, b.q_pos, b.kv_len,
        torch.empty((w.tokens, w.heads, 512), dtype=torch.float32, device=dev) if out is None
        else out,
        torch.empty((w.tokens, w.heads), dtype=torch.float32, device=dev) if lse is None else lse,
        scale=w.scale, query_counts=b.query_counts)
    out, lse = launch()
    torch.cuda.synchronize()
    assert launch.device_error() == 0
    return out, lse


def _whole(seed=41):
    lens = np.array([20000, 4097, 64, 9000], dtype=np.int64)
    w = inputs.Workload("ctx_merge", seed, 128, 576, lens, np.ones(4, np.int64), lens - 1,
                        ops.default_scale(576))
    return inputs._finish(w)


def test_single_rank_communicator_merge(cuda_device):
    w = _whole()
    full = inputs.materialize(w, cuda_device)
    order, ref_out, ref_lse = gh.oracle_tokens(full, w, range(w.tokens))
    del full
    comm = tdist.Comm(tdist.Comm.new_id(), 1, 0)
    try:
        # One rank: its partial over all pages merges to the full result.
        po, pl = _partial(w, cuda_device)
        out, lse = tdist.context_merge(comm, po, pl)
        torch.cuda.synchronize()
        assert_parity(_np(out), _np(lse), ref_out, ref_lse, label="1-rank merge")
        # The eight parts of an 8-GPU split, gathered here by hand, merge the same way.
        parts = [_partial(tdist.context_split(w, 8, r), cuda_device) for r in range(8)]
        m_out, m_lse = ops.combine_parts(torch.stack([p[0] for p in parts]),
                                         torch.stack([p[1] for p in parts]))
        torch.cuda.synchronize()
        assert_parity(_np(m_out), _np(m_lse), ref_out, ref_lse, label="8-part merge")
    finally:
        comm.destroy()


def test_single_rank_peer_merge(cuda_device):
    """The peer-memory merge on a one-rank communicator: decode into the exchange region, merge
    (no peers to wait for), twice, so the device-side step counter advances."""
    w = _whole()
    full = inputs.materialize(w, cuda_device)
    order, ref_out, ref_lse = gh.oracle_tokens(full, w, range(w.tokens))
    del full
    comm = tdist.Comm(tdist.Comm.new_id(), 1, 0)
    pm = None
    try:
        pm = tdist.PeerMerge(comm, w.tokens, w.heads)
        for step in range(2):
            _partial(w, cuda_device, pm.part_out, pm.part_lse)
            out = torch.empty((w.tokens, w.heads, 512), dtype=torch.bfloat16, device=cuda_device)
            lse = torch.empty((w.tokens, w.heads), dtype=torch.float32, device=cuda_device)
            pm.merge(out, lse)
            torch.cuda.synchronize()
            assert pm.device_error() == 0
            assert_parity(_np(out), _np(lse), ref_out, ref_lse, label=f"1-rank peer merge {step}")
    finally:
        if pm is not None:
            pm.destroy()
        comm.destroy()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    comm = None
    try:
        comm = tdist.Comm.from_process_group()
        w = _whole()
        part = tdist.context_split(w, world, rank)
        po, pl = _partial(part, dev)
        out, lse = tdist.context_merge(comm, po, pl)
        torch.cuda.synchronize()
        # The same split merged over NVLink peer memory, three steps in a row.
        pm = tdist.PeerMerge(comm, w.tokens, w.heads)
        try:
            p_out = torch.empty((w.tokens, w.heads, 512), dtype=torch.bfloat16, device=dev)
            p_lse = torch.empty((w.tokens, w.heads), dtype=torch.float32, device=dev)
            for _ in range(3):
                _partial(part, dev, pm.part_out, pm.part_lse)
                pm.merge(p_out, p_lse)
            torch.cuda.synchronize()
            flags = pm.device_error()
        finally:
            pm.destroy()
        np.savez(f"{result_path}.{rank}.npz", out=_np(out), lse=_np(lse), peer_out=_np(p_out),
                 peer_lse=_np(p_lse), peer_flags=flags)
    finally:
        if comm is not None:
            comm.destroy()
        dist.destroy_process_group()


@pytest.mark.timeout(600)
def test_two_rank_context_merge(cuda_device, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs on this box")
    import torch.multiprocessing as tmp

    result = str(tmp_path / "merged")
    tmp.start_processes(_rank_main, args=(2, _free_port(), result), nprocs=2, join=True,
                        start_method="spawn")
    w = _whole()
    full = inputs.materialize(w, cuda_device)
    order, ref_out, ref_lse = gh.oracle_tokens(full, w, range(w.tokens))
    got = [np.load(f"{result}.{r}.npz") for r in range(2)]
    for g in got:
        assert_parity(g["out"], g["lse"], ref_out, ref_lse, label="2-rank merge")
        assert int(g["peer_flags"]) == 0
        assert_parity(g["peer_out"], g["peer_lse"], ref_out, ref_lse, label="2-rank peer merge")
    np.testing.assert_array_equal(got[0]["out"], got[1]["out"])
    np.testing.assert_array_equal(got[0]["lse"], got[1]["lse"])
    np.testing.assert_array_equal(got[0]["peer_out"], got[1]["peer_out"])
