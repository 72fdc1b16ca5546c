"""Oracle (test infrastructure only): NumPy restatement of the seeded synthetic-input generator.

Nothing in the product imports this module. The product generates the same inputs with its own
C++ (host) and CUDA (device) code; tests check both against this restatement bit for bit.

The Philox word stream is the reference's (``reference/contracts/philox.md:63-75``). The
transforms below are builder-defined because the reference leaves them out of scope
(``reference/contracts/philox.md:83-87``):
  - normal ``i`` of a stream = Box-Muller on words ``2i`` and ``2i+1``:
    ``u1 = ((w0 >> 8) + 1) * 2**-24`` in ``(0, 1]``, ``u2 = (w1 >> 8) * 2**-24``,
    ``z = sqrt(-2 ln u1) * cos(2 pi u2)`` in float64, then rounded to bf16 (nearest even);
  - bounded integer ``lo + w mod (hi - lo + 1)`` from word ``i``;
  - Fisher-Yates permutation of ``P`` pages: step ``k`` (``k = 0..P-2``) swaps ``perm[i]`` and
    ``perm[j]`` with ``i = P-1-k`` and ``j = word_k mod (i+1)``.
Stream ids: q = 1, kv rows = 2, lengths = 3, page permutation = 4, prefill prefixes = 5.
Element ``(t, h, d)`` of ``q`` is normal ``(t*H + h)*D + d``; element ``d`` of the cache row of
sequence ``b`` at position ``p`` is normal ``(tok_off[b] + p)*D + d`` where ``tok_off`` is the
exclusive prefix sum of the cached lengths. Pool rows that hold no cached token are NaN.
"""

import numpy as np

from . import philox

STREAM_Q, STREAM_KV, STREAM_LEN, STREAM_PERM, STREAM_PREFIX = 1, 2, 3, 4, 5
PAGE_ROWS = 64
BF16_NAN = 0x7FC0


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round finite float64 to bf16 (nearest, ties to even) in one step; returns uint16 bits.

    The rounding acts on the float64 bit pattern (drop 45 mantissa bits with RNE), so there is
    no double rounding through float32. The rounded value has at most 8 significant bits and
    converts to float32 exactly, whose top half is the bf16 pattern.
    """
    f = np.ascontiguousarray(x, dtype=np.float64)
    b64 = f.view(np.uint64)
    # bf16 keeps 7 explicit mantissa bits; float64 has 52 -> drop 45 bits with RNE.
    drop = np.uint64(45)
    lsb = (b64 >> drop) & np.uint64(1)
    rounded = b64 + (np.uint64((1 << 44) - 1) + lsb)
    r64 = (rounded >> drop) << drop
    r = r64.view(np.float64).astype(np.float32)  # exact: r has at most 8 significant bits
    return (r.view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def bf16_to_f64(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(
        np.float32).astype(np.float64)


def normals(seed: int, stream: int, start: int, count: int) -> np.ndarray:
    """Float64 normals ``start .. start+count-1`` of a stream (before bf16 rounding)."""
    w = philox.words(seed, stream, 2 * start, 2 * count).reshape(count, 2)
    u1 = ((w[:, 0] >> np.uint32(8)).astype(np.float64) + 1.0) * 2.0**-24
    u2 = (w[:, 1] >> np.uint32(8)).astype(np.float64) * 2.0**-24
    return np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)


def normal_bf16(seed: int, stream: int, start: int, count: int) -> np.ndarray:
    return bf16_bits(normals(seed, stream, start, count))


def bounded(seed: int, stream: int, count: int, lo: int, hi: int) -> np.ndarray:
    w = philox.words(seed, stream, 0, count).astype(np.int64)
    return lo + w % (hi - lo + 1)


def lognormal_lengths(seed: int, count: int, median: float, sigma: float, lo: int, hi: int):
    z = normals(seed, STREAM_LEN, 0, count)
    return np.clip(np.rint(np.exp(np.log(median) + sigma * z)), lo, hi).astype(np.int64)


def permutation(seed: int, pages: int) -> np.ndarray:
    perm = np.arange(pages, dtype=np.int64)
    if pages > 1:
        w = philox.words(seed, STREAM_PERM, 0, pages - 1).astype(np.int64)
        for k in range(pages - 1):
            i = pages - 1 - k
            j = int(w[k] % (i + 1))
            perm[i], perm[j] = perm[j], perm[i]
    return perm


def page_tables(seed: int, kv_len, pool_pages=None):
    """Block tables drawn from a permuted pool; returns ``(page_table [S, L], pool_pages)``."""
    kv_len = np.asarray(kv_len, dtype=np.int64)
    npages = (kv_len + PAGE_ROWS - 1) // PAGE_ROWS
    total = int(npages.sum())
    if pool_pages is None:
        pool_pages = total
    assert pool_pages >= total
    perm = permutation(seed, pool_pages)
    width = max(1, int(npages.max()) if len(npages) else 1)
    table = np.zeros((len(kv_len), width), dtype=np.int32)
    off = 0
    for b, n in enumerate(npages):
        table[b, :n] = perm[off: off + n]
        off += n
    return table, pool_pages


def kv_pool(seed: int, kv_len, page_table, pool_pages: int, width: int) -> np.ndarray:
    """bf16 bit patterns of the pool ``[pool_pages * 64, width]``; unused rows are NaN."""
    kv_len = np.asarray(kv_len, dtype=np.int64)
    pool = np.full((pool_pages * PAGE_ROWS, width), BF16_NAN, dtype=np.uint16)
    tok_off = np.concatenate([[0], np.cumsum(kv_len)[:-1]]) if len(kv_len) else []
    for b, n in enumerate(kv_len):
        if n == 0:
            continue
        vals = normal_bf16(seed, STREAM_KV, int(tok_off[b]) * width, int(n) * width)
        pos = np.arange(n)
        rows = page_table[b, pos // PAGE_ROWS].astype(np.int64) * PAGE_ROWS + pos % PAGE_ROWS
        pool[rows] = vals.reshape(n, width)
    return pool


def queries(seed: int, tokens: int, heads: int, width: int) -> np.ndarray:
    return normal_bf16(seed, STREAM_Q, 0, tokens * heads * width).reshape(tokens, heads, width)
