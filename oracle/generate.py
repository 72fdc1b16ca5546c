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


class Workload:
    """Host metadata of one seeded configuration, restated without the product library.

    Mirrors the product's workload table (lengths, query counts, prefixes, page tables) so the
    CPU legs of the benchmark and the tests can rebuild a batch from the seed alone.
    """

    def __init__(self, name, seed, heads, width, kv_len, q_per_seq, prefix, scale,
                 pool_pages=None, kv_format="bf16"):
        self.name, self.seed, self.heads, self.width = name, seed, heads, width
        self.kv_len = np.asarray(kv_len, dtype=np.int64)
        self.q_per_seq = np.asarray(q_per_seq, dtype=np.int64)
        self.prefix = np.asarray(prefix, dtype=np.int64)
        self.scale = float(scale)
        self.kv_format = kv_format
        self.page_table, self.pool_pages = page_tables(seed, self.kv_len, pool_pages)
        self.token_start = np.concatenate([[0], np.cumsum(self.q_per_seq)[:-1]]).astype(np.int64)
        self.tok_off = np.concatenate([[0], np.cumsum(self.kv_len)[:-1]]).astype(np.int64)

    @property
    def sequences(self):
        return len(self.kv_len)

    @property
    def tokens(self):
        return int(self.q_per_seq.sum())

    def seq_id(self):
        return np.repeat(np.arange(self.sequences), self.q_per_seq).astype(np.int32)

    def q_pos(self):
        if not self.sequences:
            return np.zeros(0, np.int32)
        return np.concatenate([self.prefix[b] + np.arange(self.q_per_seq[b])
                               for b in range(self.sequences)]).astype(np.int32)

    def sequence_rows(self, b):
        """Float64 cache rows ``[kv_len[b], width]`` of sequence ``b`` (bf16 values)."""
        n = int(self.kv_len[b])
        return bf16_to_f64(normal_bf16(self.seed, STREAM_KV, int(self.tok_off[b]) * self.width,
                                       n * self.width)).reshape(n, self.width)

    def sequence_queries(self, b):
        """Float64 queries ``[q_per_seq[b], heads, width]`` of sequence ``b`` (bf16 values)."""
        t = int(self.q_per_seq[b])
        per = self.heads * self.width
        return bf16_to_f64(normal_bf16(self.seed, STREAM_Q, int(self.token_start[b]) * per,
                                       t * per)).reshape(t, self.heads, self.width)


def config(name, batch=None):
    """The five seeded configurations (and the FP8 decode batch), metadata only.

    ``cpu``: 4 x 1 token, 16 heads, lengths {17, 64, 200, 1000}, a 64-page pool, seed 0.
    ``decode`` / ``decode_fp8``: 64 x 1 token, 128 heads, lengths U[4096, 8192], seed 1.
    ``prefill``: 8 x 2048 new tokens over prefixes U[0, 6144] (stream 5), seed 2.
    ``longctx``: 4 x 1 token over 131072 cached rows, seed 3.
    ``mtp``: 512 x 2 tokens, lengths lognormal(median 8192, sigma 1) clipped to [256, 65536],
    seed 4.
    """
    scale = 1.0 / np.sqrt(192.0)
    if name == "cpu":
        kv = np.array([17, 64, 200, 1000], dtype=np.int64)
        return Workload("cpu_decode_h16", 0, 16, 576, kv, np.ones(4), kv - 1, scale, 64)
    if name in ("decode", "decode_fp8"):
        b = 64 if batch is None else batch
        kv = bounded(1, STREAM_LEN, b, 4096, 8192)
        if name == "decode_fp8":
            return Workload("decode_fp8_b64_h128_ctx4k-8k", 1, 128, 512, kv, np.ones(b), kv - 1,
                            0.0625, kv_format="fp8_e4m3")
        return Workload("decode_b64_h128_ctx4k-8k", 1, 128, 576, kv, np.ones(b), kv - 1, scale)
    if name == "prefill":
        b = 8 if batch is None else batch
        pre = bounded(2, STREAM_PREFIX, b, 0, 6144)
        return Workload("prefill_8x2048_prefix0-6k_h128", 2, 128, 576, pre + 2048,
                        np.full(b, 2048), pre, scale)
    if name in ("sparse", "sparse_fp8"):
        b = 64 if batch is None else batch
        kv = np.full(b, 32768, dtype=np.int64)
        return Workload(f"{name}_b{b}_h32_ctx32k_k2048", 1, 32, 512, kv, np.ones(b), kv - 1,
                        0.0625, kv_format="fp8_e4m3" if name == "sparse_fp8" else "bf16")
    if name == "longctx":
        b = 4 if batch is None else batch
        kv = np.full(b, 131072, dtype=np.int64)
        return Workload("longctx_b4_131072_h128", 3, 128, 576, kv, np.ones(b), kv - 1, scale)
    if name == "mtp":
        b = 512 if batch is None else batch
        kv = lognormal_lengths(4, b, 8192.0, 1.0, 256, 65536)
        return Workload("mtp_512x2_lognormal8k_h128", 4, 128, 576, kv, np.full(b, 2), kv - 2,
                        scale)
    raise KeyError(name)
