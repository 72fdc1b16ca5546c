"""GPU: the MLA prologue (tq_mla_prologue) through the C ABI against the float64 oracle.

Sizes are the two models' own: the reference's no-RoPE model (hidden 4096, Q rank 1536, 64 heads
of 256, 512-wide rows, bf16 and FP8 pool rows) and the 576-wide RoPE form (hidden 7168, Q rank
1536, 128 heads of 128 + 64). The projections accumulate in f32 on the device and in float64 in
the oracle, so q and the rows agree to bf16 rounding, with the tolerance written in each check;
pool rows the call does not name stay byte for byte as they were.
"""

import numpy as np
import pytest
import torch

from oracle import fp8 as ofp8
from oracle import prologue as opro
from tq_mla import _abi, ops

pytestmark = pytest.mark.gpu

PAYLOAD = {_abi.KV_BF16: 1024, _abi.KV_FP8_E4M3: 528, _abi.KV_BF16_ROPE576: 1152}
FILL = 0xA5


def _bf16(a, device):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16).to(device)


def _placement(rng, tokens, seqs, slots, pool_pages, max_pos):
    """Sequence ids, positions and a page table whose (page, row) slots are all distinct."""
    table = rng.integers(0, pool_pages, (seqs, slots)).astype(np.int32)
    seq = rng.integers(0, seqs, tokens).astype(np.int32)
    pos = np.zeros(tokens, np.int32)
    used = set()
    for t in range(tokens):
        while True:
            p = int(rng.integers(0, max_pos))
            slot = (int(table[seq[t], p // 64]), p % 64)
            if slot not in used:
                used.add(slot)
                pos[t] = p
                break
    return seq, pos, table


def _case(device, *, tokens, dm, rq, heads, dn, dr, fmt, seqs=5, slots=40, pool_pages=96,
          seed=0, bad_token=None):
    rng = np.random.default_rng(seed)
    w = dict(
        x=rng.standard_normal((tokens, dm)),
        w_qa=rng.standard_normal((rq, dm)) / np.sqrt(dm),
        q_norm=rng.uniform(0.5, 1.5, rq),
        w_qb=rng.standard_normal((heads * (dn + dr), rq)) / np.sqrt(rq),
        w_uk=rng.standard_normal((heads, dn, 512)) / np.sqrt(dn),
        w_kva=rng.standard_normal((512 + dr, dm)) / np.sqrt(dm),
        kv_norm=rng.uniform(0.5, 1.5, 512))
    dev = {k: _bf16(v, device) for k, v in w.items()}
    host = {k: v.float().cpu().numpy().astype(np.float64) for k, v in dev.items()}
    seq, pos, table = _placement(rng, tokens, seqs, slots, pool_pages, slots * 64)
    if bad_token is not None:
        seq[bad_token] = seqs                      # out of range: q produced, no row written
    row = (PAYLOAD[fmt] + 15) // 16 * 16
    pool = torch.full((pool_pages, 64, row), FILL, dtype=torch.uint8, device=device)
    flags = torch.zeros(1, dtype=torch.int32, device=device)
    q = ops.mla_prologue(dev["x"], dev["w_qa"], dev["q_norm"], dev["w_qb"], dev["w_uk"],
                         dev["w_kva"], dev["kv_norm"], torch.from_numpy(pos).to(device),
                         torch.from_numpy(seq).to(device), torch.from_numpy(table).to(device),
                         pool, heads=heads, nope_dim=dn, rope_dim=dr, kv_format=fmt, flags=flags)
    torch.cuda.synchronize()
    q_ref, kvf = opro.prologue(host["x"], host["w_qa"], host["q_norm"], host["w_qb"], host["w_uk"],
                               host["w_kva"], host["kv_norm"], pos, heads=heads, nope_dim=dn,
                               rope_dim=dr, q_eps=1e-6, kv_eps=1e-6, rope_theta=10000.0)
    pool0 = np.full((pool_pages, 64, row), FILL, np.uint8)
    pool_ref, skipped = opro.write_rows(pool0, kvf, host["kv_norm"], table, seq, pos,
                                        kv_format=fmt, kv_eps=1e-6)
    return dict(q=q.float().cpu().numpy().astype(np.float64), q_ref=q_ref,
                pool=pool.cpu().numpy(), pool_ref=pool_ref, skipped=skipped,
                flags=int(flags.item()), seq=seq, pos=pos, table=table, fmt=fmt)


def _check_q(q, q_ref):
    """Within two bf16 steps of the value plus 2^-6 of the head row's RMS, relative L2 within
    2^-8, and at least half of the values bit-equal. The device accumulates its GEMMs in f32 in
    its own order (cuBLAS's, or the projection kernel's K boxes and splits): a bf16 rounding of cq or qf that lands on the other side moves every value
    after it by ~6e-4 of the row's scale (the same chain in PyTorch's bf16 matmuls gives this
    library's bits exactly). A wrong head, transpose, sign or rotation is off by the row's scale."""
    rms = np.sqrt(np.mean(q_ref ** 2, axis=-1, keepdims=True))
    err = np.abs(q - q_ref)
    assert np.all(err <= 2.0 ** -6 * np.abs(q_ref) + 2.0 ** -6 * rms), (err / rms).max()
    assert np.linalg.norm(q - q_ref) <= 2.0 ** -8 * np.linalg.norm(q_ref)
    assert np.mean(q == q_ref) > 0.5


def _rows(r, flat):
    out = []
    for t in range(len(r["seq"])):
        if r["skipped"][t]:
            continue
        p = int(r["pos"][t])
        out.append(int(r["table"][r["seq"][t], p // 64]) * 64 + p % 64)
    return np.array(out)


def _check_rows(r):
    flat, ref = r["pool"].reshape(-1, r["pool"].shape[-1]), r["pool_ref"].reshape(-1, r["pool"].shape[-1])
    named = _rows(r, flat)
    other = np.setdiff1d(np.arange(flat.shape[0]), named)
    np.testing.assert_array_equal(flat[other], ref[other])          # untouched rows
    pay = PAYLOAD[r["fmt"]]
    np.testing.assert_array_equal(flat[named, pay:], ref[named, pay:])  # padding untouched
    if r["fmt"] == _abi.KV_FP8_E4M3:
        got, want = ofp8.dequant_rows(flat[named]), ofp8.dequant_rows(ref[named])
        scale_g = flat[named, 512:528].copy().view("<f4")
        scale_w = ref[named, 512:528].copy().view("<f4")
        np.testing.assert_allclose(scale_g, scale_w, rtol=2.0 ** -7)
        # one E4M3 step (2^-3 of the value) when the bf16 input or the scale moved by one step
        amax = np.repeat(scale_w * 448.0, 128, axis=1)
        assert np.all(np.abs(got - want) <= 2.0 ** -3 * np.abs(want) + 2.0 ** -9 * amax)
        assert np.mean(flat[named, :512] == ref[named, :512]) > 0.97
    else:
        w = pay // 2
        got = (flat[named, :pay].copy().view(np.uint16).astype(np.uint32) << 16).view(np.float32)
        want = (ref[named, :pay].copy().view(np.uint16).astype(np.uint32) << 16).view(np.float32)
        got, want = got.reshape(-1, w).astype(np.float64), want.reshape(-1, w).astype(np.float64)
        rms = np.sqrt(np.mean(want ** 2, axis=-1, keepdims=True))
        # a projected value one bf16 step away is two steps away after the norm's two roundings
        assert np.all(np.abs(got - want) <= 2.0 ** -6 * np.abs(want) + 2.0 ** -9 * rms)
        assert np.mean(got == want) > 0.97


@pytest.mark.parametrize("fmt", [_abi.KV_BF16, _abi.KV_FP8_E4M3])
def test_no_rope_model_sizes(cuda_device, fmt):
    r = _case(cuda_device, tokens=48, dm=4096, rq=1536, heads=64, dn=256, dr=0, fmt=fmt, seed=1)
    assert r["q"].shape == (48, 64, 512)
    _check_q(r["q"], r["q_ref"])
    _check_rows(r)
    assert r["flags"] == 0


def test_rope_576_sizes_and_large_positions(cuda_device):
    r = _case(cuda_device, tokens=40, dm=7168, rq=1536, heads=128, dn=128, dr=64,
              fmt=_abi.KV_BF16_ROPE576, slots=2048, pool_pages=160, seed=2)
    assert r["pos"].max() > 60000                  # RoPE angles far from zero
    assert r["q"].shape == (40, 128, 576)
    _check_q(r["q"], r["q_ref"])
    _check_rows(r)


@pytest.mark.parametrize("tokens,dm", [(1, 1000), (33, 1536), (128, 1000), (129, 1536)])
def test_token_counts_and_ragged_tiles(cuda_device, tokens, dm):
    """Decode batches of 1 to 128 tokens take the weight-streaming projections (token tiles of
    16, 48 and 128 rows; a hidden size that ends inside a 64-wide chunk; Q rank and head widths
    that end inside a 128-row weight tile); 129 tokens take the library GEMMs."""
    r = _case(cuda_device, tokens=tokens, dm=dm, rq=320, heads=12, dn=128, dr=64,
              fmt=_abi.KV_BF16_ROPE576, slots=64, pool_pages=200, seed=10 + tokens)
    assert r["q"].shape == (tokens, 12, 576)
    _check_q(r["q"], r["q_ref"])
    _check_rows(r)
    assert r["flags"] == 0


def test_out_of_range_token_flags_and_keeps_its_query(cuda_device):
    r = _case(cuda_device, tokens=12, dm=512, rq=256, heads=8, dn=128, dr=64,
              fmt=_abi.KV_BF16_ROPE576, seed=3, bad_token=5)
    assert r["skipped"][5] and r["skipped"].sum() == 1
    assert r["flags"] == _abi.DEV_SEQ_RANGE
    _check_q(r["q"], r["q_ref"])
    _check_rows(r)


def test_graph_replay_matches_the_direct_call(cuda_device):
    """The prologue captured in a CUDA graph replays to the same bits as a direct call."""
    rng = np.random.default_rng(9)
    tokens, dm, rq, heads, dn = 16, 1024, 512, 16, 256
    dev = dict(x=_bf16(rng.standard_normal((tokens, dm)), cuda_device),
               w_qa=_bf16(rng.standard_normal((rq, dm)) / 32, cuda_device),
               q_norm=_bf16(np.ones(rq), cuda_device),
               w_qb=_bf16(rng.standard_normal((heads * dn, rq)) / 22, cuda_device),
               w_uk=_bf16(rng.standard_normal((heads, dn, 512)) / 16, cuda_device),
               w_kva=_bf16(rng.standard_normal((512, dm)) / 32, cuda_device),
               kv_norm=_bf16(np.ones(512), cuda_device))
    pos = torch.arange(tokens, dtype=torch.int32, device=cuda_device)
    seq = torch.zeros(tokens, dtype=torch.int32, device=cuda_device)
    table = torch.arange(4, dtype=torch.int32, device=cuda_device).reshape(1, 4)
    pool = torch.zeros((4, 64, 528), dtype=torch.uint8, device=cuda_device)
    q = torch.empty((tokens, heads, 512), dtype=torch.bfloat16, device=cuda_device)
    args = [dev[k] for k in ("x", "w_qa", "q_norm", "w_qb", "w_uk", "w_kva", "kv_norm")]
    pro = ops.MlaPrologue(*args, pos, seq, table, pool, q, heads=heads, nope_dim=dn, rope_dim=0,
                          kv_format=_abi.KV_FP8_E4M3)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        pro(stream=s)
    s.synchronize()
    q1, pool1 = q.clone(), pool.clone()
    q.zero_(); pool.zero_()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        pro(stream=s)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(q, q1) and torch.equal(pool, pool1)
