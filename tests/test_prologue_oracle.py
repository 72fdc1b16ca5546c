"""The prologue oracle, CPU only: its absorption pinned to the reference's MLA fixture cases, its
RMSNorm against the model's formula run in torch, RoPE properties, and the cache write routed
through the writer oracle."""

from pathlib import Path

import numpy as np
import torch

from oracle import kv_write as okw
from oracle import mla as omla
from oracle import prologue as opro

GOLDEN = Path(__file__).parent / "golden"


def _rel_l2(a, b):
    d = np.linalg.norm(np.asarray(a) - np.asarray(b))
    n = np.linalg.norm(np.asarray(b))
    return d / n if n else d


def test_absorption_reproduces_the_reference_fixture_outputs():
    """Absorbing the fixture's pre-absorption queries with ``opro.absorb`` and attending over the
    latent rows in absorbed form reproduces the reference's expected outputs (the fixtures hold the
    unabsorbed ``q`` and ``w_uk``; the expected values come from the pinned Transformers model),
    including the model-width case (Dn 256, R 512)."""
    g = np.load(GOLDEN / "mla_upstream.npz")
    keys = sorted({k.split("__")[0] for k in g.files})
    assert "glm_width_b0" in keys
    for key in keys:
        q, lat = g[f"{key}__q"], g[f"{key}__latent"]
        w_uk, w_uv, mask = g[f"{key}__w_uk"], g[f"{key}__w_uv"], g[f"{key}__mask"]
        scale = float(g[f"{key}__scale"])
        exp = g[f"{key}__expected"]
        q_abs = opro.absorb(q, w_uk)
        assert q_abs.shape == (q.shape[0], q.shape[1], lat.shape[1])
        for t in range(q.shape[0]):
            rows = lat[mask[t]]
            if len(rows) == 0:
                np.testing.assert_array_equal(exp[t], 0)
                continue
            o_lat, _ = omla.identity_core(q_abs[t], rows, scale, lat.shape[1])
            out = np.einsum("hvr,hr->hv", w_uv, o_lat)
            assert _rel_l2(out, exp[t]) <= 1e-12, (key, t)


def test_rms_norm_follows_the_model_rounding_points():
    """``weight * (x.float() * rsqrt(mean(x^2) + eps)).to(bf16)`` in torch, the model's RMSNorm
    for bf16 activations: the oracle agrees on nearly every value and never by more than one bf16
    step (torch's rsqrt and its f32 mean round differently from the float64 oracle)."""
    rng = np.random.default_rng(11)
    x = torch.from_numpy(rng.standard_normal((64, 1536)) * 3.0).to(torch.bfloat16)
    w = torch.from_numpy(rng.uniform(0.2, 2.0, 1536)).to(torch.bfloat16)
    xf = x.float()
    h = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)
    want = (w * h.to(torch.bfloat16)).float().numpy().astype(np.float64)
    got = opro.rms_norm(x.float().numpy(), w.float().numpy(), 1e-6)
    assert np.mean(got == want) > 0.99
    np.testing.assert_allclose(got, want, rtol=2 ** -7, atol=0)


def test_rope_rotates_pairs_and_composes():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((7, 3, 64))
    pos = np.array([0, 1, 5, 63, 64, 4095, 2 ** 20])
    y = opro.rope_exact(x, pos, 10000.0)
    np.testing.assert_allclose(y[0], x[0], rtol=0, atol=0)        # position 0 is the identity
    pair_norm = lambda v: np.hypot(v[..., 0::2], v[..., 1::2])
    np.testing.assert_allclose(pair_norm(y), pair_norm(x), rtol=1e-12)
    # rotating by a then by b equals rotating by a + b (pair 0 turns by exactly pos radians)
    a, b = np.array([3, 70, 1000]), np.array([11, 5, 77])
    xa = opro.rope_exact(x[:3], a, 10000.0)
    np.testing.assert_allclose(opro.rope_exact(xa, b, 10000.0),
                               opro.rope_exact(x[:3], a + b, 10000.0), atol=1e-9)
    z = np.zeros((1, 1, 64)); z[..., 0] = 1.0
    r = opro.rope_exact(z, np.array([2]), 10000.0)
    np.testing.assert_allclose(r[0, 0, :2], [np.cos(2.0), np.sin(2.0)], atol=1e-15)
    # the last pair turns slowest: theta^(-62/64)
    z = np.zeros((1, 1, 64)); z[..., 62] = 1.0
    r = opro.rope_exact(z, np.array([1000]), 10000.0)
    ang = 1000 * 10000.0 ** (-62 / 64)
    np.testing.assert_allclose(r[0, 0, 62:], [np.cos(ang), np.sin(ang)], atol=1e-12)


def _small_weights(rng, dm, rq, heads, dn, dr):
    def bf(a):
        return torch.from_numpy(a).to(torch.bfloat16).float().numpy().astype(np.float64)
    return dict(
        x=bf(rng.standard_normal((9, dm))),
        w_qa=bf(rng.standard_normal((rq, dm)) / np.sqrt(dm)),
        q_norm=bf(rng.uniform(0.5, 1.5, rq)),
        w_qb=bf(rng.standard_normal((heads * (dn + dr), rq)) / np.sqrt(rq)),
        w_uk=bf(rng.standard_normal((heads, dn, 512)) / np.sqrt(dn)),
        w_kva=bf(rng.standard_normal((512 + dr, dm)) / np.sqrt(dm)),
        kv_norm=bf(rng.uniform(0.5, 1.5, 512)))


def test_prologue_shapes_and_bf16_outputs():
    rng = np.random.default_rng(2)
    for heads, dn, dr in ((4, 256, 0), (3, 128, 64)):
        w = _small_weights(rng, 64, 48, heads, dn, dr)
        pos = np.arange(9) * 37
        q, kvf = opro.prologue(**w, pos=pos, heads=heads, nope_dim=dn, rope_dim=dr, q_eps=1e-6,
                               kv_eps=1e-6, rope_theta=10000.0)
        assert q.shape == (9, heads, 512 + dr) and kvf.shape == (9, 512 + dr)
        for v in (q, kvf):
            assert np.array_equal(opro.bf16(v), v)                 # every value is a bf16
        # the absorbed part is the absorption of the projected nope part, to bf16 rounding
        cq = opro.rms_norm(opro.bf16(w["x"] @ w["w_qa"].T), w["q_norm"], 1e-6)
        qf = opro.bf16(cq @ w["w_qb"].T).reshape(9, heads, dn + dr)
        np.testing.assert_array_equal(q[:, :, :512], opro.bf16(opro.absorb(qf[:, :, :dn],
                                                                           w["w_uk"])))
        if dr:
            np.testing.assert_array_equal(q[:, :, 512:], opro.rope(qf[:, :, dn:], pos, 10000.0))


def test_rows_are_the_writer_with_its_norm():
    rng = np.random.default_rng(4)
    w = _small_weights(rng, 64, 48, 2, 128, 0)
    pos = np.array([0, 1, 2, 64, 65, 127, 128, 129, 300])
    seq = np.array([0, 0, 0, 0, 0, 0, 1, 1, 2])
    table = np.array([[3, 0, 9], [5, 1, 2], [4, 7, 8]], np.int32)
    _, kvf = opro.prologue(**w, pos=pos, heads=2, nope_dim=128, rope_dim=0, q_eps=1e-6,
                           kv_eps=1e-6, rope_theta=10000.0)
    pool = np.zeros((10, 64, 544), np.uint8)
    got, skipped = opro.write_rows(pool, kvf, w["kv_norm"], table, seq, pos, kv_format=1,
                                   kv_eps=1e-6)
    assert skipped.tolist() == [False] * 8 + [True]                # pos 300 is past 3 pages
    normed = okw.rms_norm_rows(opro.bf16_bits(kvf), opro.bf16_bits(w["kv_norm"]), 1e-6)
    want = okw.row_bytes(normed, 1)
    flat = got.reshape(-1, 544)
    for t in range(8):
        row = table[seq[t], pos[t] // 64] * 64 + pos[t] % 64
        np.testing.assert_array_equal(flat[row, :528], want[t])
    # the writer's f32 norm and the float64 model norm agree to one bf16 step
    f32 = (normed.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    np.testing.assert_allclose(f32, opro.rms_norm(kvf, w["kv_norm"], 1e-6), rtol=2 ** -7, atol=0)
