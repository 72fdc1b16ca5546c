"""Oracle (test infrastructure only): float64 NumPy restatement of the absorbed MLA core.

Nothing in the product imports this module. Tests, ``__graft_entry__.smoke()`` and the CPU
baseline leg of ``bench.py`` use it as the checker for the CUDA kernels.

Restated from ``reference/src/tq_reference/mla_attention.py``:
  - ``mla_attention_core``   follows :135-169 (per token: absorb, score, shift by max, exp,
                             normalise by the shifted weights, project, lse = m + log(sum w));
  - ``split_kv_b``           follows :87-107 (per-head interleaved key then value rows);
  - validation fragments     follow :41-84 and :110-132 (float64, finite, consistent shapes).
Paged dense decode (``paged_attention``) is the build's dense-paged extension: each query token
``t`` attends to cache positions ``[0, min(kv_len[seq_id[t]], q_pos[t] + 1))``, gathered through
the page table, with identity key absorption (``w_uk = I``) and value projection ``[I_512 | 0]``.
With those weights the general core reduces exactly (multiplications by one and additions of
zero) to ``identity_core`` below; a test checks the two agree.
"""

import numpy as np

PAGE_ROWS = 64


class MlaError(ValueError):
    """Invalid input to, or arithmetic overflow in, the oracle."""


def _require(name, value, dtype, ndim):
    if not isinstance(value, np.ndarray):
        raise MlaError(f"{name} must be a numpy.ndarray")
    if value.dtype != dtype:
        raise MlaError(f"{name} must have dtype {np.dtype(dtype).name}")
    if value.ndim != ndim:
        raise MlaError(f"{name} must have {ndim} dimensions")
    if 0 in value.shape:
        raise MlaError(f"{name} has an empty dimension")
    return value


def _finite(stage, value):
    if not np.isfinite(value).all():
        raise MlaError(f"overflow in {stage}")


def _scale(scale):
    if isinstance(scale, bool) or not isinstance(scale, (int, float, np.integer, np.floating)):
        raise MlaError("scale must be a real scalar")
    value = float(scale)
    if not (np.isfinite(value) and value > 0):
        raise MlaError("scale must be finite and > 0")
    return value


def split_kv_b(w_kv_b, *, num_heads, qk_nope_head_dim, v_head_dim):
    """Split packed ``[H*(Dn+Dv), R]`` into ``(w_uk [H,Dn,R], w_uv [H,Dv,R])``."""
    w = _require("w_kv_b", w_kv_b, np.float64, 2)
    if w.shape[0] != num_heads * (qk_nope_head_dim + v_head_dim):
        raise MlaError("w_kv_b rows must equal num_heads * (qk_nope_head_dim + v_head_dim)")
    per_head = w.reshape(num_heads, qk_nope_head_dim + v_head_dim, w.shape[1])
    return (
        np.ascontiguousarray(per_head[:, :qk_nope_head_dim, :]),
        np.ascontiguousarray(per_head[:, qk_nope_head_dim:, :]),
    )


def mla_attention_core(q, latent, w_uk, w_uv, mask, *, scale):
    """General absorbed MLA for one sequence: returns ``(out [T,H,Dv], out_latent [T,H,R], lse)``."""
    _require("q", q, np.float64, 3)
    _require("latent", latent, np.float64, 2)
    _require("w_uk", w_uk, np.float64, 3)
    _require("w_uv", w_uv, np.float64, 3)
    _require("mask", mask, np.bool_, 2)
    t_count, heads, key_dim = q.shape
    keys, rank = latent.shape
    if w_uk.shape != (heads, key_dim, rank) or w_uv.shape[0::2] != (heads, rank):
        raise MlaError("shape mismatch")
    if mask.shape != (t_count, keys):
        raise MlaError("shape mismatch")
    for name, arr in (("q", q), ("latent", latent), ("w_uk", w_uk), ("w_uv", w_uv)):
        if not np.isfinite(arr).all():
            raise MlaError(f"{name} contains non-finite values")
    scale = _scale(scale)
    value_dim = w_uv.shape[1]
    out = np.zeros((t_count, heads, value_dim))
    out_latent = np.zeros((t_count, heads, rank))
    lse = np.full((t_count, heads), -np.inf)
    with np.errstate(all="ignore"):
        for t in range(t_count):
            sel = np.flatnonzero(mask[t])
            if sel.size == 0:
                continue
            rows = latent[sel]
            q_abs = np.einsum("hd,hdr->hr", q[t], w_uk)
            _finite("absorbed query", q_abs)
            s = (q_abs @ rows.T) * scale
            _finite("score", s)
            m = s.max(axis=1, keepdims=True)
            w = np.exp(s - m)
            total = w.sum(axis=1, keepdims=True)
            lat = (w / total) @ rows
            _finite("latent output", lat)
            o = np.einsum("hvr,hr->hv", w_uv, lat)
            _finite("output", o)
            out_latent[t] = lat
            out[t] = o
            lse[t] = m[:, 0] + np.log(total[:, 0])
    return out, out_latent, lse


def identity_core(q_t, rows, scale, value_dim):
    """One query token with identity absorption: ``q_t [H,D]``, ``rows [n,D]`` float64.

    Same operation order as ``mla_attention_core`` with ``w_uk = I`` and ``w_uv = [I|0]``.
    Returns ``(out [H,value_dim], lse [H])``; ``n == 0`` gives zeros and ``-inf``.
    """
    heads = q_t.shape[0]
    if rows.shape[0] == 0:
        return np.zeros((heads, value_dim)), np.full(heads, -np.inf)
    with np.errstate(all="ignore"):
        s = (q_t @ rows.T) * scale
        m = s.max(axis=1, keepdims=True)
        w = np.exp(s - m)
        total = w.sum(axis=1, keepdims=True)
        lat = (w / total) @ rows[:, :value_dim]
        lse = m[:, 0] + np.log(total[:, 0])
    return lat, lse


def visible_length(seq_id, q_pos, kv_len, t):
    """Keys visible to query token ``t``: ``min(kv_len[s], q_pos[t] + 1)``, 0 when invalid."""
    s = int(seq_id[t])
    if s < 0 or s >= len(kv_len):
        return 0
    return max(0, min(int(kv_len[s]), int(q_pos[t]) + 1))


def gather_rows(pool_rows, page_table_row, n):
    """Rows ``[0, n)`` of one sequence: pool row index ``page * 64 + slot`` for each position."""
    pos = np.arange(n)
    idx = page_table_row[pos // PAGE_ROWS].astype(np.int64) * PAGE_ROWS + pos % PAGE_ROWS
    return pool_rows[idx]


def row_byte_offsets(page_table_row, n, row_stride):
    """Byte offset into the pool of each visible position (the kernel's page indexing)."""
    pos = np.arange(n, dtype=np.int64)
    return (page_table_row[pos // PAGE_ROWS].astype(np.int64) * PAGE_ROWS + pos % PAGE_ROWS) * int(
        row_stride
    )


def paged_attention(q, pool_rows, page_table, seq_id, q_pos, kv_len, *, scale, value_dim=512,
                    tokens=None):
    """Dense paged decode/prefill oracle in float64.

    ``q [T,H,D]`` and ``pool_rows [P*64, D]`` are float64 (bf16 values widened exactly).
    Returns ``(out [T,H,value_dim], lse [T,H])`` for the selected ``tokens`` (default all).
    """
    scale = _scale(scale)
    t_all = range(q.shape[0]) if tokens is None else tokens
    out = np.zeros((len(t_all), q.shape[1], value_dim))
    lse = np.full((len(t_all), q.shape[1]), -np.inf)
    for i, t in enumerate(t_all):
        n = visible_length(seq_id, q_pos, kv_len, t)
        rows = gather_rows(pool_rows, page_table[int(seq_id[t])], n) if n else pool_rows[:0]
        out[i], lse[i] = identity_core(q[t], rows, scale, value_dim)
    return out, lse


def sparse_entries(idx_row, k_len, q_pos, kv_len):
    """Valid entries of one token's index row, in order (``docs/TEST-PLAN.md:199``): entry j is
    valid iff ``j < k_len`` and ``0 <= idx[j] <= q_pos`` and ``idx[j] < kv_len``."""
    k = max(0, min(int(k_len), len(idx_row)))
    v = np.asarray(idx_row[:k], dtype=np.int64)
    return v[(v >= 0) & (v <= int(q_pos)) & (v < int(kv_len))]


def sparse_attention(q, pool_rows, page_table, seq_id, q_pos, kv_len, idx, k_len, *, scale,
                     value_dim=512):
    """Sparse top-k paged decode oracle in float64 (the DSA form of ``SmlaSpec``,
    ``contracts.rs:196-200``): token ``t`` attends to the rows of its valid index entries, i.e.
    ``mla_attention_core`` with the mask of those positions. Rows are gathered in entry order
    (an entry listed twice would count twice; the contract's indices are unique per token)."""
    scale = _scale(scale)
    t_count, heads = q.shape[0], q.shape[1]
    out = np.zeros((t_count, heads, value_dim))
    lse = np.full((t_count, heads), -np.inf)
    for t in range(t_count):
        s = int(seq_id[t])
        if s < 0 or s >= len(kv_len):
            continue
        v = sparse_entries(idx[t], k_len[t], q_pos[t], kv_len[s])
        rows_idx = page_table[s][v // PAGE_ROWS].astype(np.int64) * PAGE_ROWS + v % PAGE_ROWS
        out[t], lse[t] = identity_core(q[t], pool_rows[rows_idx], scale, value_dim)
    return out, lse


def combine_partials(partial_out, partial_lse):
    """Log-sum-exp merge of split results along axis 0.

    ``partial_out [k, ..., Dv]`` holds outputs normalised over each part and ``partial_lse
    [k, ...]`` their natural-log lse. A row whose parts are all ``-inf`` yields zeros and
    ``-inf`` with no NaN. A NaN part (a NaN in one of its visible rows) makes the merged row NaN,
    as the unsplit attention over the same rows is (anomaly positions match the single pass).
    """
    nan_part = np.isnan(partial_lse)
    m = np.where(nan_part, -np.inf, partial_lse).max(axis=0)
    finite = np.isfinite(m)
    safe_m = np.where(finite, m, 0.0)
    with np.errstate(invalid="ignore", over="ignore"):
        w = np.where(np.isneginf(partial_lse), 0.0, np.exp(partial_lse - safe_m))
        total = w.sum(axis=0)
        denom = np.where(total == 0, 1.0, total)
        out = np.where((total == 0)[..., None], 0.0,
                       (w[..., None] * partial_out).sum(0) / denom[..., None])
        lse = np.where(total == 0, -np.inf, safe_m + np.log(denom))
    return out, lse
