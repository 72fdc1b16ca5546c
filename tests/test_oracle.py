"""The oracle is pinned before it is trusted.

- Its MLA core reproduces the reference's pinned-Transformers fixtures (rel-L2 <= 1e-12, the
  reference's own bar: reference/tests/test_mla_acceptance.py:106-135).
- Its paged, identity-absorbed path reproduces outputs computed by the reference's own
  ``mla_attention_core`` on the same seeded inputs (tests/golden/paged_cases.npz).
- The seeded generator reproduces the recorded input hashes; the product's host generator
  (C-ABI Philox) gives the same lengths, permutations and block tables, bit for bit.
- The split-KV partition covers every page of every token exactly once; a log-sum-exp merge of
  split results equals the unsplit result.
- A planted mistake in the oracle is caught by the parity check (the checker can fail).
"""

import hashlib

import numpy as np
import pytest

from conftest import GOLDEN, assert_parity
from oracle import generate as ogen
from oracle import mla as omla
from oracle import schedule as osched
from tq_mla import inputs


def _rel_l2(a, b):
    n = np.linalg.norm(b)
    return np.linalg.norm(a - b) / n if n else np.abs(a - b).max()


def test_core_matches_upstream_transformers_fixtures():
    g = np.load(GOLDEN / "mla_upstream.npz")
    keys = sorted({k.split("__")[0] for k in g.files})
    assert len(keys) == 6  # 5 cases, asym_multihead has two batch entries
    for key in keys:
        out, lat, lse = omla.mla_attention_core(
            g[f"{key}__q"], g[f"{key}__latent"], g[f"{key}__w_uk"], g[f"{key}__w_uv"],
            g[f"{key}__mask"], scale=float(g[f"{key}__scale"]))
        exp = g[f"{key}__expected"]
        assert out.shape == exp.shape
        assert _rel_l2(out, exp) <= 1e-12, key
        for t in range(exp.shape[0]):
            for h in range(exp.shape[1]):
                if np.linalg.norm(exp[t, h]) == 0:
                    np.testing.assert_array_equal(out[t, h], 0)
                    assert np.isneginf(lse[t, h])
                else:
                    assert _rel_l2(out[t, h], exp[t, h]) <= 1e-12, (key, t, h)


def test_split_kv_b_matches_the_reference_split_of_the_fixture_weights():
    """The oracle's split of each fixture's packed kv_b weight equals the reference's split
    (w_uk, w_uv stored by make_golden.py from reference/src/tq_reference/mla_attention.py:87-107),
    and the packing checks of :95-101 reject a wrong row count."""
    g = np.load(GOLDEN / "mla_upstream.npz")
    keys = sorted(k[: -len("__w_kv_b")] for k in g.keys() if k.endswith("__w_kv_b"))
    assert len(keys) >= 5
    for key in keys:
        heads, dn, dv = (int(x) for x in g[f"{key}__kv_b_dims"])
        w_uk, w_uv = omla.split_kv_b(g[f"{key}__w_kv_b"], num_heads=heads, qk_nope_head_dim=dn,
                                     v_head_dim=dv)
        np.testing.assert_array_equal(w_uk, g[f"{key}__w_uk"], err_msg=key)
        np.testing.assert_array_equal(w_uv, g[f"{key}__w_uv"], err_msg=key)
        with pytest.raises(omla.MlaError):
            omla.split_kv_b(g[f"{key}__w_kv_b"][:-1], num_heads=heads, qk_nope_head_dim=dn,
                            v_head_dim=dv)


def test_identity_core_equals_general_core_with_identity_weights():
    rng = np.random.default_rng(0)
    h, d, n = 4, 576, 37
    q = rng.standard_normal((1, h, d))
    rows = rng.standard_normal((n, d))
    w_uk = np.broadcast_to(np.eye(d), (h, d, d)).copy()
    w_uv = np.broadcast_to(np.eye(512, d), (h, 512, d)).copy()
    mask = np.ones((1, n), bool)
    out, _, lse = omla.mla_attention_core(q, rows, w_uk, w_uv, mask, scale=192 ** -0.5)
    o2, l2 = omla.identity_core(q[0], rows, 192 ** -0.5, 512)
    np.testing.assert_allclose(o2, out[0], rtol=0, atol=1e-13)
    np.testing.assert_allclose(l2, lse[0], rtol=0, atol=1e-13)


@pytest.mark.parametrize("name", ["cfg1_decode_h16", "mtp_h32", "nope512_h32"])
def test_paged_oracle_reproduces_reference_outputs(name):
    g = np.load(GOLDEN / "paged_cases.npz")
    seed, heads, per_seq, width, pool_pages = (int(x) for x in g[f"{name}__meta"])
    lens = g[f"{name}__kv_len"]
    table, pp = ogen.page_tables(seed, lens, pool_pages)
    np.testing.assert_array_equal(table, g[f"{name}__page_table"])
    pool = ogen.kv_pool(seed, lens, table, pp, width)
    q = ogen.queries(seed, len(lens) * per_seq, heads, width)
    assert hashlib.sha256(pool.tobytes()).hexdigest() == str(g[f"{name}__pool_sha256"])
    assert hashlib.sha256(q.tobytes()).hexdigest() == str(g[f"{name}__q_sha256"])
    out, lse = omla.paged_attention(ogen.bf16_to_f64(q), ogen.bf16_to_f64(pool), table,
                                    g[f"{name}__seq_id"], g[f"{name}__q_pos"], lens,
                                    scale=float(g[f"{name}__scale"]))
    ref_out, ref_lse = g[f"{name}__out"], g[f"{name}__lse"]
    assert _rel_l2(out, ref_out) <= 1e-12
    np.testing.assert_allclose(lse, ref_lse, rtol=0, atol=1e-12 * max(1, np.abs(ref_lse).max()))


def test_unused_pool_rows_are_nan_and_never_read():
    g = np.load(GOLDEN / "paged_cases.npz")
    lens = g["cfg1_decode_h16__kv_len"]
    table, pp = ogen.page_tables(0, lens, 64)
    pool = ogen.bf16_to_f64(ogen.kv_pool(0, lens, table, pp, 576))
    used = np.zeros(pp * 64, bool)
    for b, n in enumerate(lens):
        pos = np.arange(n)
        used[table[b, pos // 64].astype(int) * 64 + pos % 64] = True
    assert np.isnan(pool[~used]).all() and np.isfinite(pool[used]).all()
    assert (~used).sum() == 64 * 64 - lens.sum()


@pytest.mark.parametrize("name", ["cpu", "decode", "prefill", "longctx", "mtp"])
def test_product_host_generator_matches_oracle(name):
    w = inputs.config(name)
    if name == "decode":
        np.testing.assert_array_equal(w.kv_len, ogen.bounded(1, ogen.STREAM_LEN, 64, 4096, 8192))
    if name == "prefill":
        np.testing.assert_array_equal(w.prefix,
                                      ogen.bounded(2, ogen.STREAM_PREFIX, 8, 0, 6144))
    if name == "mtp":
        np.testing.assert_array_equal(w.kv_len, ogen.lognormal_lengths(4, 512, 8192.0, 1.0, 256,
                                                                       65536))
    table, pp = ogen.page_tables(w.seed, w.kv_len, 64 if name == "cpu" else None)
    assert pp == w.pool_pages
    np.testing.assert_array_equal(table, w.extra["page_table"])


def test_config_shapes_match_the_workloads():
    assert inputs.config("decode").tokens == 64
    w = inputs.config("prefill")
    assert w.tokens == 8 * 2048 and (w.kv_len == w.prefix + 2048).all()
    assert (inputs.config("longctx").kv_len == 131072).all()
    w = inputs.config("mtp")
    assert w.tokens == 1024 and w.kv_len.min() >= 256 and w.kv_len.max() <= 65536
    v = w.visible()
    np.testing.assert_array_equal(v[0::2] + 1, v[1::2])  # causal between the two tokens


def test_bf16_rounding_is_nearest_even():
    x = np.array([1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -1.0 - 2 ** -8, 1.0 + 2 ** -8 + 2 ** -40,
                  3.0e-3, -7.5])
    bits = ogen.bf16_bits(x)
    back = ogen.bf16_to_f64(bits)
    np.testing.assert_array_equal(back[:4], [1.0, 1.0 + 2 ** -6, -1.0, 1.0 + 2 ** -7])
    assert abs(back[4] - 3.0e-3) <= 2 ** -8 * 3.0e-3 and back[5] == -7.5


@pytest.mark.parametrize("pairs", [1, 2, 7, 74])
def test_partition_covers_every_page_once(pairs):
    rng = np.random.default_rng(pairs)
    n_vis = rng.integers(0, 3000, size=97)
    n_vis[::11] = 0
    meta = osched.partition(n_vis, pairs)
    covered = {u: np.zeros(int(p), int) for u, p in enumerate(meta["pages"])}
    slots = set()
    for c in range(pairs):
        for u, p0, n, slot in osched.segments(meta, c):
            covered[u][p0:p0 + n] += 1
            if slot >= 0:
                assert slot not in slots
                slots.add(slot)
    for u, cov in covered.items():
        assert (cov == 1).all(), u
    assert meta["slots"] <= 2 * pairs
    assert set(meta["empty_units"]) == set(np.flatnonzero(n_vis == 0))


def test_lse_merge_of_splits_equals_unsplit():
    rng = np.random.default_rng(3)
    q = rng.standard_normal((8, 576))
    rows = rng.standard_normal((1000, 576))
    full_o, full_l = omla.identity_core(q, rows, 0.07, 512)
    cuts = [0, 1, 64, 500, 999, 1000]
    parts = [omla.identity_core(q, rows[a:b], 0.07, 512) for a, b in zip(cuts[:-1], cuts[1:])]
    parts.append((np.zeros((8, 512)), np.full(8, -np.inf)))  # an empty split
    o, l_ = omla.combine_partials(np.stack([p[0] for p in parts]), np.stack([p[1] for p in parts]))
    np.testing.assert_allclose(o, full_o, rtol=0, atol=1e-13)
    np.testing.assert_allclose(l_, full_l, rtol=0, atol=1e-12)
    o, l_ = omla.combine_partials(np.zeros((2, 8, 512)), np.full((2, 8), -np.inf))
    assert (o == 0).all() and np.isneginf(l_).all()


def test_lse_merge_keeps_a_nan_split_nan():
    """A NaN in one split's visible rows makes the merged row NaN, like the unsplit pass."""
    rng = np.random.default_rng(4)
    q = rng.standard_normal((4, 576))
    rows = rng.standard_normal((300, 576))
    rows[170, 9] = np.nan
    full_o, full_l = omla.identity_core(q, rows, 0.07, 512)
    assert np.isnan(full_o).all() and np.isnan(full_l).all()
    cuts = [0, 128, 256, 300]
    parts = [omla.identity_core(q, rows[a:b], 0.07, 512) for a, b in zip(cuts[:-1], cuts[1:])]
    parts.append((np.zeros((4, 512)), np.full(4, -np.inf)))
    o, l_ = omla.combine_partials(np.stack([p[0] for p in parts]), np.stack([p[1] for p in parts]))
    assert np.isnan(o).all() and np.isnan(l_).all()


def test_planted_mistake_in_the_oracle_is_caught():
    """The parity check fails when the oracle uses the wrong scale (the checker has teeth)."""
    g = np.load(GOLDEN / "paged_cases.npz")
    name = "cfg1_decode_h16"
    lens = g[f"{name}__kv_len"]
    table, pp = ogen.page_tables(0, lens, 64)
    pool = ogen.bf16_to_f64(ogen.kv_pool(0, lens, table, pp, 576))
    q = ogen.bf16_to_f64(ogen.queries(0, 4, 16, 576))
    args = (q, pool, table, g[f"{name}__seq_id"], g[f"{name}__q_pos"], lens)
    good = omla.paged_attention(*args, scale=192 ** -0.5)
    bad = omla.paged_attention(*args, scale=512 ** -0.5)
    assert_parity(good[0], good[1], g[f"{name}__out"], g[f"{name}__lse"])
    with pytest.raises(AssertionError):
        assert_parity(bad[0], bad[1], g[f"{name}__out"], g[f"{name}__lse"])


@pytest.mark.parametrize("name", ["sparse_h32", "sparse_k2051"])
def test_sparse_oracle_matches_reference_core_with_the_valid_mask(name):
    """The sparse oracle against ``mla_attention_core`` run by the reference on the same seeded
    inputs with each token's valid-position mask (tests/golden/sparse_cases.npz)."""
    g = np.load(GOLDEN / "sparse_cases.npz")
    seed, heads, width, pool_pages = (int(x) for x in g[f"{name}__meta"])
    lens = g[f"{name}__kv_len"]
    table, pp = ogen.page_tables(seed, lens, pool_pages)
    np.testing.assert_array_equal(table, g[f"{name}__page_table"])
    pool = ogen.kv_pool(seed, lens, table, pp, width)
    tokens = int(g[f"{name}__per_seq"].sum())
    q = ogen.queries(seed, tokens, heads, width)
    assert hashlib.sha256(pool.tobytes()).hexdigest() == str(g[f"{name}__pool_sha256"])
    assert hashlib.sha256(q.tobytes()).hexdigest() == str(g[f"{name}__q_sha256"])
    out, lse = omla.sparse_attention(ogen.bf16_to_f64(q), ogen.bf16_to_f64(pool), table,
                                     g[f"{name}__seq_id"], g[f"{name}__q_pos"], lens,
                                     g[f"{name}__idx"], g[f"{name}__k_len"],
                                     scale=float(g[f"{name}__scale"]))
    np.testing.assert_allclose(out, g[f"{name}__out"], rtol=0, atol=1e-12)
    np.testing.assert_allclose(lse, g[f"{name}__lse"], rtol=0, atol=1e-12)
