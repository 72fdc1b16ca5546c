"""Oracle (test infrastructure only): the MLA prologue, token activations to absorbed queries and
cache rows.

Nothing in the product imports this module; tests use it to check ``tq_mla_prologue``.

The reference plans "a fused MLA prologue (q_a -> norm -> q_b -> absorb; kv_a -> norm -> cache
write)" (``docs/DEV-PLAN.md:116``, ``docs/research/glm-5.md:602``) and ships no implementation of
it; the pieces it does define are restated here:

- the key absorption ``q_abs = w_uk[h].T @ q[t, h]`` of
  ``reference/src/tq_reference/mla_attention.py:150`` (pinned against the reference's own MLA
  fixture cases in the tests);
- RMSNorm as the model applies it to ``q_a`` and ``kv_a`` (squares in f32, the normalised value
  rounded to bf16 before the weight multiplies it; ``docs/reviews/2026-09-19-design-review.md:13``);
- the cache write of ``oracle/kv_write.py`` (row formats of ``docs/HOST-CONTRACTS.md:122-123``).

The reference's model has no RoPE (``docs/research/glm-5.md:163-167``); for 576-wide rows this
build defines RoPE on pairs (2i, 2i + 1) rotated by ``pos * theta^(-2i / 64)``.

Arithmetic: products and sums in float64, rounded to bf16 at the points where the device rounds
(after each projection, after the norm, after the weight, after RoPE). The device accumulates its
GEMMs in f32 in an order of its own, so q agrees to within bf16 rounding, not bit for bit; the
cache write is bit-exact given the same bf16 projection.
"""

import numpy as np

from oracle import kv_write as okw
from oracle.fp8 import bf16_round

LATENT = 512
ROPE = 64


def bf16(x):
    """float64 values rounded (through f32) to the nearest bf16, returned as float64."""
    with np.errstate(over="ignore", invalid="ignore"):
        return bf16_round(np.asarray(x, dtype=np.float64).astype(np.float32))


def bf16_bits(x):
    """bf16 bit patterns (uint16) of values that are already bf16."""
    return (np.asarray(x, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def absorb(q_nope, w_uk):
    """``q_abs[t, h] = w_uk[h].T @ q_nope[t, h]`` (mla_attention.py:150): ``q_nope [T, H, Dn]``,
    ``w_uk [H, Dn, R]`` -> ``[T, H, R]`` in float64."""
    return np.einsum("thd,hdr->thr", np.asarray(q_nope, np.float64), np.asarray(w_uk, np.float64))


def rms_norm(x, weight, eps):
    """The model's RMSNorm of each row of ``x`` (bf16 values): ``bf16(w * bf16(x * r))`` with
    ``r = 1 / sqrt(mean(x^2) + eps)``, the mean taken in float64."""
    x = np.asarray(x, np.float64)
    r = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    return bf16(bf16(x * r) * np.asarray(weight, np.float64))


def rope_exact(x, pos, theta):
    """RoPE of the last axis (64 values, pairs (2i, 2i + 1)) at positions ``pos`` (broadcast over
    the leading axes of ``x`` after the first), in float64 without rounding."""
    x = np.asarray(x, np.float64)
    i = np.arange(ROPE // 2, dtype=np.float64)
    freq = np.exp2(-2.0 * i / ROPE * np.log2(theta))
    p = np.asarray(pos, np.float64).reshape((-1,) + (1,) * (x.ndim - 1))
    angle = np.fmod(p * freq, 2.0 * np.pi)
    c, s = np.cos(angle), np.sin(angle)
    x0, x1 = x[..., 0::2], x[..., 1::2]
    out = np.empty_like(x)
    out[..., 0::2] = x0 * c - x1 * s
    out[..., 1::2] = x0 * s + x1 * c
    return out


def rope(x, pos, theta):
    """``rope_exact`` rounded to bf16, as the device stores it."""
    return bf16(rope_exact(x, pos, theta))


def prologue(x, w_qa, q_norm, w_qb, w_uk, w_kva, kv_norm, pos, *, heads, nope_dim, rope_dim,
             q_eps, kv_eps, rope_theta):
    """The prologue of every token (all arrays bf16 values as float64 or float32).

    Returns ``(q, kvf)``: ``q`` float64 ``[T, H, 512 + Dr]`` (bf16 values) and ``kvf`` float64
    ``[T, 512 + Dr]``, the projected cache row before its norm (RoPE part already rotated), which
    ``write_rows`` turns into pool rows.
    """
    x = np.asarray(x, np.float64)
    t = x.shape[0]
    dn, dr = nope_dim, rope_dim
    cq = bf16(x @ np.asarray(w_qa, np.float64).T)
    cqn = rms_norm(cq, q_norm, q_eps)
    qf = bf16(cqn @ np.asarray(w_qb, np.float64).T).reshape(t, heads, dn + dr)
    q = np.empty((t, heads, LATENT + dr))
    q[:, :, :LATENT] = bf16(absorb(qf[:, :, :dn], w_uk))
    if dr:
        q[:, :, LATENT:] = rope(qf[:, :, dn:], pos, rope_theta)
    return q, cache_rows(x, w_kva, pos, rope_dim=dr, rope_theta=rope_theta)


def cache_rows(x, w_kva, pos, *, rope_dim, rope_theta):
    """``kvf = bf16(x . w_kva^T)`` with its RoPE part rotated (``[T, 512 + Dr]``, bf16 values):
    the cache half of the prologue before the writer's norm."""
    kvf = bf16(np.asarray(x, np.float64) @ np.asarray(w_kva, np.float64).T)
    if rope_dim:
        kvf[:, LATENT:] = rope(kvf[:, LATENT:], pos, rope_theta)
    return kvf


def write_rows(pool_u8, kvf, kv_norm, page_table, seq_id, pos, *, kv_format, kv_eps):
    """The cache write of ``kvf`` (the device writer's norm and FP8 rule, bit for bit): returns
    ``(pool, skipped)`` as ``oracle.kv_write.write`` does."""
    return okw.write(pool_u8, bf16_bits(kvf), page_table, seq_id, pos, kv_format,
                     norm_weight_bits=bf16_bits(kv_norm), norm_eps=kv_eps)
