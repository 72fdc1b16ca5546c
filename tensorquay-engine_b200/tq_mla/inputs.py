"""Seeded synthetic workloads: the five paged-MLA configurations and their device tensors.

Host metadata (lengths, page permutation, block tables) comes from the library's Philox stream
(``tq_philox_words``, the reference's stream: reference/contracts/philox.md:63-75); device data
(queries, cache rows) comes from ``tq_gen_normal_bf16`` / ``tq_gen_kv_pool``. The transforms are
builder-defined (the reference leaves normal transforms and permutations out of scope,
reference/contracts/philox.md:83-87):
  - normal ``i`` of a stream: Box-Muller on words ``2i, 2i+1``,
    ``u1 = ((w0 >> 8) + 1) 2^-24``, ``u2 = (w1 >> 8) 2^-24``, ``z = sqrt(-2 ln u1) cos(2 pi u2)``
    in float64, rounded to bf16 (nearest even);
  - bounded integer: ``lo + word_i mod (hi - lo + 1)``;
  - permutation of ``P`` pages: Fisher-Yates, step ``k`` swaps ``i = P-1-k`` with
    ``word_k mod (i+1)``.
Streams: q 1, cache rows 2, lengths 3, permutation 4, prefill prefixes 5.
"""

import ctypes
from dataclasses import dataclass, field

import numpy as np

from ._abi import lib, raise_for

PAGE_ROWS = 64
STREAM_Q, STREAM_KV, STREAM_LEN, STREAM_PERM, STREAM_PREFIX = 1, 2, 3, 4, 5


def philox_words(seed, stream, start, count):
    out = np.zeros(max(count, 1), dtype=np.uint32)
    raise_for(lib.tq_philox_words(seed, stream, start,
                                  out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)), count))
    return out[:count]


def host_normals(seed, stream, start, count):
    w = philox_words(seed, stream, 2 * start, 2 * count).reshape(count, 2)
    u1 = ((w[:, 0] >> np.uint32(8)).astype(np.float64) + 1.0) * 2.0 ** -24
    u2 = (w[:, 1] >> np.uint32(8)).astype(np.float64) * 2.0 ** -24
    return np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)


def uniform_lengths(seed, count, lo, hi, stream=STREAM_LEN):
    w = philox_words(seed, stream, 0, count).astype(np.int64)
    return lo + w % (hi - lo + 1)


def lognormal_lengths(seed, count, median, sigma, lo, hi):
    z = host_normals(seed, STREAM_LEN, 0, count)
    return np.clip(np.rint(np.exp(np.log(median) + sigma * z)), lo, hi).astype(np.int64)


def permutation(seed, pages):
    perm = np.arange(pages, dtype=np.int64)
    if pages > 1:
        w = philox_words(seed, STREAM_PERM, 0, pages - 1).astype(np.int64)
        for k in range(pages - 1):
            i = pages - 1 - k
            j = int(w[k] % (i + 1))
            perm[i], perm[j] = perm[j], perm[i]
    return perm


def page_tables(seed, kv_len, pool_pages=None):
    kv_len = np.asarray(kv_len, dtype=np.int64)
    npages = (kv_len + PAGE_ROWS - 1) // PAGE_ROWS
    total = int(npages.sum())
    pool_pages = total if pool_pages is None else int(pool_pages)
    if pool_pages < total:
        raise ValueError("pool smaller than the cached pages")
    perm = permutation(seed, pool_pages)
    width = max(1, int(npages.max()) if len(npages) else 1)
    table = np.zeros((len(kv_len), width), dtype=np.int32)
    off = 0
    for b, n in enumerate(npages):
        table[b, :n] = perm[off:off + n]
        off += n
    return table, pool_pages


@dataclass
class Workload:
    """One paged-MLA batch: host metadata plus the global token/sequence numbering."""

    name: str
    seed: int
    heads: int
    width: int
    kv_len: np.ndarray          # [S] cached length per sequence
    q_per_seq: np.ndarray       # [S] query tokens per sequence
    prefix: np.ndarray          # [S] position of the first query token
    scale: float
    pool_pages: int = None
    seq_global: np.ndarray = None   # [S] global sequence index (for data streams)
    token_global: np.ndarray = None  # [S] global index of each sequence's first query token
    tok_off_global: np.ndarray = None  # [S] global cached-token offset of each sequence
    extra: dict = field(default_factory=dict)

    @property
    def sequences(self):
        return len(self.kv_len)

    @property
    def tokens(self):
        return int(self.q_per_seq.sum())

    def seq_id(self):
        return np.repeat(np.arange(self.sequences), self.q_per_seq).astype(np.int32)

    def q_pos(self):
        return np.concatenate([self.prefix[b] + np.arange(self.q_per_seq[b])
                               for b in range(self.sequences)]).astype(np.int32) \
            if self.sequences else np.zeros(0, np.int32)

    def visible(self):
        """Keys visible per query token: ``min(kv_len, q_pos + 1)``."""
        return np.minimum(self.kv_len[self.seq_id()], self.q_pos().astype(np.int64) + 1)

    def flops(self):
        return 2.0 * self.heads * (self.width + 512) * float(self.visible().sum())

    def bytes(self):
        """Algorithmic bytes: each cached row once, q, out, lse, block tables and lengths."""
        rows = float(self.kv_len.sum()) * self.extra.get("kv_row_bytes", self.width * 2)
        pages = float(((self.kv_len + PAGE_ROWS - 1) // PAGE_ROWS).sum())
        t = self.tokens
        return rows + t * self.heads * (self.width * 2 + 1024 + 4) + 4 * pages + 4 * self.sequences


def _finish(w: Workload, pool_pages=None):
    s = w.sequences
    if w.seq_global is None:
        w.seq_global = np.arange(s)
    if w.token_global is None:
        w.token_global = np.concatenate([[0], np.cumsum(w.q_per_seq)[:-1]]).astype(np.int64)
    if w.tok_off_global is None:
        w.tok_off_global = np.concatenate([[0], np.cumsum(w.kv_len)[:-1]]).astype(np.int64)
    table, w.pool_pages = page_tables(w.seed, w.kv_len, pool_pages)
    w.extra["page_table"] = table
    return w


def config(name, *, batch=None):
    """The reference configurations (seeded): ``cpu``, ``decode``, ``prefill``, ``longctx``, ``mtp``."""
    scale = 1.0 / np.sqrt(192.0)
    if name == "cpu":
        kv = np.array([17, 64, 200, 1000], dtype=np.int64)
        w = Workload("cpu_decode_h16", 0, 16, 576, kv, np.ones(4, np.int64), kv - 1, scale)
        return _finish(w, pool_pages=64)
    if name in ("sparse", "sparse_fp8"):
        # Sparse top-k decode in the reference's SMLA-P-001 shape: sequences x 1 token, 32 heads,
        # 32K cached positions each, bf16 (1024-byte) or FP8 (528 of 544 bytes) rows; the top-k
        # index sets are drawn by the bench (2048 valid of 2051 entries per token).
        b = 64 if batch is None else batch
        kv = np.full(b, 32768, dtype=np.int64)
        w = Workload(f"{name}_b{b}_h32_ctx32k_k2048", 1, 32, 512, kv, np.ones(b, np.int64),
                     kv - 1, 0.0625)
        if name == "sparse_fp8":
            w.extra["kv_format"] = "fp8_e4m3"
            w.extra["kv_row_bytes"] = FP8_ROW_PAYLOAD
        return _finish(w)
    if name == "decode_fp8":
        # The decode batch with FP8 E4M3 rows (512 codes + 4 f32 scales; no RoPE part, q width
        # 512, the format's fixed scale 1/16).
        b = 64 if batch is None else batch
        kv = uniform_lengths(1, b, 4096, 8192)
        w = Workload("decode_fp8_b64_h128_ctx4k-8k", 1, 128, 512, kv, np.ones(b, np.int64),
                     kv - 1, 0.0625)
        w.extra["kv_format"] = "fp8_e4m3"
        w.extra["kv_row_bytes"] = FP8_ROW_PAYLOAD
        return _finish(w)
    if name == "decode":
        b = 64 if batch is None else batch
        kv = uniform_lengths(1, b, 4096, 8192)
        return _finish(Workload("decode_b64_h128_ctx4k-8k", 1, 128, 576, kv,
                                np.ones(b, np.int64), kv - 1, scale))
    if name == "prefill":
        b = 8 if batch is None else batch
        pre = uniform_lengths(2, b, 0, 6144, stream=STREAM_PREFIX)
        kv = pre + 2048
        return _finish(Workload("prefill_8x2048_prefix0-6k_h128", 2, 128, 576, kv,
                                np.full(b, 2048, np.int64), pre, scale))
    if name == "longctx":
        b = 4 if batch is None else batch
        kv = np.full(b, 131072, dtype=np.int64)
        return _finish(Workload("longctx_b4_131072_h128", 3, 128, 576, kv,
                                np.ones(b, np.int64), kv - 1, scale))
    if name == "mtp":
        b = 512 if batch is None else batch
        kv = lognormal_lengths(4, b, 8192.0, 1.0, 256, 65536)
        return _finish(Workload("mtp_512x2_lognormal8k_h128", 4, 128, 576, kv,
                                np.full(b, 2, np.int64), kv - 2, scale))
    raise KeyError(name)


def shard(w: Workload, ranks: int, rank: int) -> Workload:
    """Token-balanced (longest-first greedy) assignment of whole sequences to ``ranks`` devices.

    Each device owns the pages of its sequences; data keeps its global stream offsets, so a
    sequence has the same contents whichever device holds it.
    """
    cost = w.kv_len * w.q_per_seq
    order = np.argsort(-cost, kind="stable")
    load = np.zeros(ranks)
    owner = np.zeros(w.sequences, dtype=np.int64)
    for b in order:
        r = int(np.argmin(load))
        owner[b] = r
        load[r] += cost[b]
    mine = np.flatnonzero(owner == rank)
    tok_global = np.concatenate([[0], np.cumsum(w.q_per_seq)[:-1]]).astype(np.int64)
    tok_off = np.concatenate([[0], np.cumsum(w.kv_len)[:-1]]).astype(np.int64)
    sub = Workload(w.name, w.seed, w.heads, w.width, w.kv_len[mine], w.q_per_seq[mine],
                   w.prefix[mine], w.scale, seq_global=mine, token_global=tok_global[mine],
                   tok_off_global=tok_off[mine])
    return _finish(sub)


@dataclass
class DeviceBatch:
    q: "torch.Tensor"
    kv: "torch.Tensor"
    page_table: "torch.Tensor"
    seq_id: "torch.Tensor"
    q_pos: "torch.Tensor"
    kv_len: "torch.Tensor"
    query_counts: list


def _gen_q(w: Workload, dev, q_seed=None):
    import torch

    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    q = torch.empty((w.tokens, w.heads, w.width), dtype=torch.bfloat16, device=dev)
    per_tok = w.heads * w.width
    local = 0
    for b in range(w.sequences):
        n = int(w.q_per_seq[b]) * per_tok
        if n:
            raise_for(lib.tq_gen_normal_bf16(ctypes.c_void_p(q.data_ptr() + 2 * local * per_tok),
                                             n, q_seed if q_seed is not None else w.seed,
                                             STREAM_Q, int(w.token_global[b]) * per_tok, stream))
        local += int(w.q_per_seq[b])
    return q


def materialize(w: Workload, device, *, row_stride=None, q_seed=None):
    """Allocate and fill the device tensors of ``w`` with the seeded generator."""
    import torch

    if w.extra.get("kv_format") == "fp8_e4m3":
        return materialize_fp8(w, device, row_stride=row_stride or 544, q_seed=q_seed)
    dev = torch.device(device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    width = w.width
    row_stride = row_stride or width * 2
    q = _gen_q(w, dev, q_seed)
    pool_bytes = max(1, w.pool_pages) * PAGE_ROWS * row_stride
    kv_raw = torch.empty(pool_bytes, dtype=torch.uint8, device=dev)
    kv = kv_raw[: w.pool_pages * PAGE_ROWS * row_stride].view(w.pool_pages, PAGE_ROWS, row_stride)
    table = torch.from_numpy(w.extra["page_table"]).to(dev)
    kv_len = torch.from_numpy(w.kv_len.astype(np.int32)).to(dev)
    tok_off = torch.from_numpy(w.tok_off_global.astype(np.int64)).to(dev)
    raise_for(lib.tq_gen_kv_pool(ctypes.c_void_p(kv_raw.data_ptr()), w.pool_pages, row_stride,
                                 width, ctypes.c_void_p(table.data_ptr()), table.shape[1],
                                 ctypes.c_void_p(kv_len.data_ptr()),
                                 ctypes.c_void_p(tok_off.data_ptr()), w.sequences, w.seed, stream))
    kv_view = kv[:, :, : width * 2].view(torch.bfloat16) if row_stride == width * 2 else kv
    return DeviceBatch(
        q=q,
        kv=kv_view,
        page_table=table,
        seq_id=torch.from_numpy(w.seq_id()).to(dev),
        q_pos=torch.from_numpy(w.q_pos()).to(dev),
        kv_len=kv_len,
        query_counts=[int(c) for c in w.q_per_seq],
    )


FP8_ROW_PAYLOAD = 528


def used_rows(w: Workload):
    """Boolean ``[pool_pages * 64]``: pool rows that hold a cached position of some sequence."""
    used = np.zeros(max(1, w.pool_pages) * PAGE_ROWS, dtype=bool)
    table = w.extra["page_table"]
    for b in range(w.sequences):
        n = int(w.kv_len[b])
        pos = np.arange(n)
        used[table[b, pos // PAGE_ROWS].astype(np.int64) * PAGE_ROWS + pos % PAGE_ROWS] = True
    return used


def materialize_fp8(w: Workload, device, *, row_stride=544, q_seed=None, poison=True):
    """Device tensors of ``w`` with FP8 E4M3 rows ``uint8 [P, 64, row_stride]``.

    q is the seeded bf16 generator's (width 512). Each cached position's 512 latent values are
    drawn N(0, 1) from a torch generator seeded with ``w.seed`` and quantized per 128-value tile
    with scale = amax / 448 (round to nearest even, the format's largest finite magnitude is
    448). With ``poison``, rows that hold no cached position carry NaN codes and NaN scales, so a
    kernel that read them would produce NaN.
    """
    import torch

    assert w.width == 512 and row_stride >= FP8_ROW_PAYLOAD and row_stride % 16 == 0
    dev = torch.device(device)
    q = _gen_q(w, dev, q_seed)
    rows_total = max(1, w.pool_pages) * PAGE_ROWS
    pool = torch.zeros((rows_total, row_stride), dtype=torch.uint8, device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(int(w.seed) * 7919 + 17)
    chunk = 1 << 16
    for r0 in range(0, rows_total, chunk):
        r1 = min(rows_total, r0 + chunk)
        x = torch.randn((r1 - r0, 4, 128), generator=gen, device=dev, dtype=torch.float32)
        amax = x.abs().amax(dim=2, keepdim=True).clamp_min(1e-30)
        scale = amax / 448.0
        codes = (x / scale).clamp(-448.0, 448.0).to(torch.float8_e4m3fn).view(torch.uint8)
        pool[r0:r1, :512] = codes.reshape(r1 - r0, 512)
        pool[r0:r1, 512:528] = scale.reshape(r1 - r0, 4).contiguous().view(torch.uint8)
    if poison:
        unused = torch.from_numpy(~used_rows(w)).to(dev)
        pool[unused, :512] = 0x7F
        nan = torch.full((1, 4), float("nan"), dtype=torch.float32, device=dev).view(torch.uint8)
        pool[unused, 512:528] = nan
    kv = pool[: w.pool_pages * PAGE_ROWS].view(w.pool_pages, PAGE_ROWS, row_stride)
    table = torch.from_numpy(w.extra["page_table"]).to(dev)
    return DeviceBatch(
        q=q,
        kv=kv,
        page_table=table,
        seq_id=torch.from_numpy(w.seq_id()).to(dev),
        q_pos=torch.from_numpy(w.q_pos()).to(dev),
        kv_len=torch.from_numpy(w.kv_len.astype(np.int32)).to(dev),
        query_counts=[int(c) for c in w.q_per_seq],
    )
