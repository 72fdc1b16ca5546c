"""Multi-device host logic on CPU with the gloo backend (world size 2).

- Request sharding is a partition of the sequences, balanced by tokens, identical on every rank.
- The context split of a long decode covers every position exactly once, page-aligned; each
  rank's partial (computed by the oracle) gathered over gloo and merged by log-sum-exp equals
  the single-device result.
- The communicator id travels from rank 0 to every rank through a gloo group unchanged.
"""

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as tmp

from oracle import generate as ogen
from oracle import mla as omla
from tq_mla import dist as tdist
from tq_mla import inputs


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_request_sharding_partitions_and_balances():
    w = inputs.config("mtp", batch=64)
    owners = []
    for world in (2, 4, 8):
        shards = [inputs.shard(w, world, r) for r in range(world)]
        got = np.sort(np.concatenate([s.seq_global for s in shards]))
        np.testing.assert_array_equal(got, np.arange(w.sequences))
        loads = np.array([(s.kv_len * s.q_per_seq).sum() for s in shards])
        assert loads.max() - loads.min() <= (w.kv_len * w.q_per_seq).max()
        for s in shards:
            # contents keep their global offsets
            full_off = np.concatenate([[0], np.cumsum(w.kv_len)[:-1]])
            np.testing.assert_array_equal(s.tok_off_global, full_off[s.seq_global])
        owners.append(shards)


def test_context_ranges_cover_each_position_once():
    for n in (1, 63, 64, 65, 131072, 131071):
        for world in (1, 2, 3, 8):
            r = tdist.context_ranges(n, world)
            assert r[0][0] == 0 and r[-1][1] == n
            for (a, b), (c, d) in zip(r[:-1], r[1:]):
                assert b == c and a % 64 == 0
            assert sum(b - a for a, b in r) == n


def _rank_main(rank, world, port, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        lens = np.array([700, 1000, 64], dtype=np.int64)
        full = inputs.Workload("ctx", 3, 16, 576, lens, np.ones(3, np.int64), lens - 1,
                               192 ** -0.5)
        full = inputs._finish(full)
        part = tdist.context_split(full, world, rank)
        # This rank's partial, from its own pool (oracle compute stands in for the device).
        pool = ogen.bf16_to_f64(ogen.kv_pool(part.seed, part.kv_len, part.extra["page_table"],
                                             part.pool_pages, 576)) if part.pool_pages else None
        # kv_pool numbers rows from a local offset; rebuild with the global offsets instead.
        rows = np.full((max(part.pool_pages, 1) * 64, 576), np.nan)
        for b, n in enumerate(part.kv_len):
            vals = ogen.bf16_to_f64(ogen.normal_bf16(part.seed, ogen.STREAM_KV,
                                                     int(part.tok_off_global[b]) * 576, int(n) * 576))
            pos = np.arange(n)
            rows[part.extra["page_table"][b, pos // 64].astype(int) * 64 + pos % 64] = \
                vals.reshape(n, 576)
        del pool
        q = ogen.bf16_to_f64(ogen.queries(full.seed, full.tokens, full.heads, 576))
        out, lse = omla.paged_attention(q, rows, part.extra["page_table"], part.seq_id(),
                                        part.q_pos(), part.kv_len, scale=part.scale)
        # Host-side stand-in for the device all-gather: each rank's partial reaches every rank.
        g_out = [torch.empty(out.shape, dtype=torch.float64) for _ in range(world)]
        g_lse = [torch.empty(lse.shape, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(g_out, torch.from_numpy(out))
        dist.all_gather(g_lse, torch.from_numpy(lse))
        merged = omla.combine_partials(torch.stack(g_out).numpy(), torch.stack(g_lse).numpy())
        if rank == 0:
            np.savez(result_path, out=merged[0], lse=merged[1])
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world", [2])
def test_context_split_gather_merge_equals_single_device(tmp_path, world):
    result = tmp_path / "merged.npz"
    tmp.start_processes(_rank_main, args=(world, _free_port(), str(result)), nprocs=world,
                        join=True, start_method="spawn")
    got = np.load(result)
    lens = np.array([700, 1000, 64], dtype=np.int64)
    table, pp = ogen.page_tables(3, lens)
    pool = ogen.bf16_to_f64(ogen.kv_pool(3, lens, table, pp, 576))
    q = ogen.bf16_to_f64(ogen.queries(3, 3, 16, 576))
    ref_out, ref_lse = omla.paged_attention(q, pool, table, np.arange(3), lens - 1, lens,
                                            scale=192 ** -0.5)
    np.testing.assert_allclose(got["out"], ref_out, rtol=0, atol=1e-12)
    np.testing.assert_allclose(got["lse"], ref_lse, rtol=0, atol=1e-12)


def _id_rank_main(rank, world, port, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        # The id that tdist.Comm.from_process_group sends (raw bytes, NUL bytes included).
        box = [bytes(range(128)) if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        assert box[0] == bytes(range(128))
        if rank == world - 1:
            open(result_path, "w").write("ok")
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_communicator_id_reaches_every_rank(tmp_path):
    result = tmp_path / "id.txt"
    tmp.start_processes(_id_rank_main, args=(2, _free_port(), str(result)), nprocs=2, join=True,
                        start_method="spawn")
    assert result.read_text() == "ok"


def test_comm_entry_points_refuse_bad_arguments():
    """Argument checks of the C entry points need no GPU and no NCCL."""
    import ctypes

    from tq_mla import _abi

    assert _abi.lib.tq_comm_unique_id(None) == 100
    cid = _abi.TqCommId()
    h = ctypes.c_void_p()
    assert _abi.lib.tq_comm_init(ctypes.byref(cid), 2, 2, ctypes.byref(h)) == 100
    assert _abi.lib.tq_comm_init(ctypes.byref(cid), 0, 0, ctypes.byref(h)) == 100
    assert _abi.lib.tq_mla_context_merge(None, None, None) == 100
    assert _abi.lib.tq_comm_destroy(None) == 100 and _abi.lib.tq_comm_abort(None) == 100
