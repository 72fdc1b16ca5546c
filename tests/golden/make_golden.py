"""Regenerate the committed golden fixtures from the reference checkout.

Run from the repository root, in a container where the reference is mounted:

    python tests/golden/make_golden.py /root/reference

It writes, under ``tests/golden/``:
  - ``philox-v1/{blocks,streams,uniform}.tsv``: the reference's Random123 known-answer vectors,
    copied byte for byte after checking each file's SHA-256 against the reference manifest;
  - ``mla_upstream.npz``: the reference's pinned-Transformers MLA fixture cases
    (``reference/tests/fixtures/transformers_mla_770e4c40_{core,glm_width}.json``), decoded to
    float64 arrays: per case the query, latent rows, split key/value expansions, mask, scale and
    the upstream SDPA output;
  - ``paged_cases.npz``: paged bf16 cases whose inputs come from the seeded generator and whose
    expected ``out``/``lse`` come from the reference's own ``mla_attention_core``, imported from
    the checkout and called with identity key absorption and ``[I_512 | 0]`` value projection;
  - ``sparse_cases.npz``: sparse top-k cases on the same kind of seeded inputs, with index rows
    drawn here (stored in the file) that mix valid entries with -1, positions past q_pos or
    kv_len, extreme values and stale padding after k_len; the expected ``out``/``lse`` come
    from ``mla_attention_core`` with the mask of each token's valid positions
    (``docs/TEST-PLAN.md:199``).
Nothing at test time reads the reference checkout; the tests read only these files.
"""

import base64
import hashlib
import json
import shutil
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from oracle import generate  # noqa: E402  (the generator's restatement defines the inputs)

PAGED_CASES = {
    # name: (seed, heads, kv_len list, queries per sequence, kv_format, pool pages or None)
    "cfg1_decode_h16": (0, 16, [17, 64, 200, 1000], 1, "rope576", 64),
    "mtp_h32": (4, 32, [65, 130], 2, "rope576", None),
    "nope512_h32": (5, 32, [1, 63, 129], 1, "nope512", None),
}


def _array(record):
    dtype = np.dtype(record["dtype"])
    raw = base64.b64decode(record["b64"], validate=True)
    return np.frombuffer(raw, dtype=dtype).reshape(tuple(record["shape"])).astype(
        dtype.newbyteorder("=")
    )


def copy_philox(ref: Path):
    src = ref / "tests/fixtures/philox-v1"
    manifest = json.loads((src / "manifest.json").read_text())
    dst = HERE / "philox-v1"
    dst.mkdir(exist_ok=True)
    for name, info in manifest["files"].items():
        digest = hashlib.sha256((src / name).read_bytes()).hexdigest()
        assert digest == info["sha256"], name
        shutil.copyfile(src / name, dst / name)
    (dst / "SHA256SUMS").write_text(
        "".join(f"{info['sha256']}  {name}\n" for name, info in manifest["files"].items())
    )


def upstream_cases(ref: Path):
    sys.path.insert(0, str(ref / "reference/src"))
    from tq_reference import mla_attention

    out = {}
    for fixture in ("core", "glm_width"):
        path = ref / f"reference/tests/fixtures/transformers_mla_770e4c40_{fixture}.json"
        data = json.loads(path.read_text())
        for case in data["cases"]:
            dims = case["dims"]
            w_kv_b = _array(case["inputs"]["kv_b_proj_weight"]).astype(np.float64)
            w_uk, w_uv = mla_attention.split_kv_b(
                w_kv_b,
                num_heads=dims["num_heads"],
                qk_nope_head_dim=dims["qk_nope_head_dim"],
                v_head_dim=dims["v_head_dim"],
            )
            scale = float(_array(case["scale"]["value"]).item())
            q = _array(case["inputs"]["q"]).astype(np.float64)
            latent = _array(case["inputs"]["latent"]).astype(np.float64)
            mask = _array(case["upstream"]["mask"])
            expected = _array(case["upstream"]["output"]).astype(np.float64)
            for b in range(dims["batch"]):
                key = f"{case['name']}_b{b}"
                out[f"{key}__q"] = np.ascontiguousarray(q[b].transpose(1, 0, 2))
                out[f"{key}__latent"] = np.ascontiguousarray(latent[b, 0])
                out[f"{key}__w_uk"] = w_uk
                out[f"{key}__w_uv"] = w_uv
                # The packed weight and its head dims, for checking the oracle's split_kv_b
                # against the reference's split of the same weight (w_uk, w_uv above).
                out[f"{key}__w_kv_b"] = w_kv_b
                out[f"{key}__kv_b_dims"] = np.array([dims["num_heads"],
                                                     dims["qk_nope_head_dim"],
                                                     dims["v_head_dim"]])
                out[f"{key}__mask"] = np.ascontiguousarray(mask[b, 0])
                out[f"{key}__scale"] = np.array(scale)
                out[f"{key}__expected"] = np.ascontiguousarray(expected[b])
    np.savez_compressed(HERE / "mla_upstream.npz", **out)


def paged_cases(ref: Path):
    sys.path.insert(0, str(ref / "reference/src"))
    from tq_reference import mla_attention

    out = {}
    for name, (seed, heads, lens, per_seq, fmt, pool) in PAGED_CASES.items():
        width = 576 if fmt == "rope576" else 512
        scale = 192 ** -0.5 if fmt == "rope576" else 0.0625
        lens = np.array(lens, dtype=np.int64)
        table, pool_pages = generate.page_tables(seed, lens, pool)
        pool_bits = generate.kv_pool(seed, lens, table, pool_pages, width)
        tokens = len(lens) * per_seq
        q_bits = generate.queries(seed, tokens, heads, width)
        seq_id = np.repeat(np.arange(len(lens)), per_seq).astype(np.int32)
        q_pos = np.concatenate([lens[b] - per_seq + np.arange(per_seq) for b in range(len(lens))])
        rows = generate.bf16_to_f64(pool_bits)
        q = generate.bf16_to_f64(q_bits)
        w_uk = np.broadcast_to(np.eye(width), (heads, width, width)).copy()
        w_uv = np.broadcast_to(np.eye(512, width), (heads, 512, width)).copy()
        exp_out = np.zeros((tokens, heads, 512))
        exp_lse = np.zeros((tokens, heads))
        for b in range(len(lens)):
            pos = np.arange(lens[b])
            latent = rows[table[b, pos // 64].astype(np.int64) * 64 + pos % 64]
            t0 = b * per_seq
            mask = np.zeros((per_seq, lens[b]), dtype=bool)
            for i in range(per_seq):
                mask[i, : q_pos[t0 + i] + 1] = True
            res = mla_attention.mla_attention_core(
                q[t0 : t0 + per_seq], latent, w_uk, w_uv, mask, scale=scale
            )
            exp_out[t0 : t0 + per_seq] = res.out
            exp_lse[t0 : t0 + per_seq] = res.lse
        out[f"{name}__meta"] = np.array([seed, heads, per_seq, width, pool_pages])
        out[f"{name}__kv_len"] = lens
        out[f"{name}__page_table"] = table
        out[f"{name}__seq_id"] = seq_id
        out[f"{name}__q_pos"] = q_pos.astype(np.int32)
        out[f"{name}__scale"] = np.array(scale)
        out[f"{name}__q_sha256"] = np.array(hashlib.sha256(q_bits.tobytes()).hexdigest())
        out[f"{name}__pool_sha256"] = np.array(hashlib.sha256(pool_bits.tobytes()).hexdigest())
        out[f"{name}__out"] = exp_out
        out[f"{name}__lse"] = exp_lse
    np.savez_compressed(HERE / "paged_cases.npz", **out)


SPARSE_CASES = {
    # name: (seed, heads, kv_len list, queries per sequence, K)
    "sparse_h32": (6, 32, [700, 64, 1500, 3000], [1, 2, 1, 3], 300),
    "sparse_k2051": (8, 32, [1, 65, 2047], [1, 1, 4], 2051),
}


def sparse_cases(ref: Path):
    sys.path.insert(0, str(ref / "reference/src"))
    from tq_reference import mla_attention

    out = {}
    for name, (seed, heads, lens, per, k) in SPARSE_CASES.items():
        width, scale = 512, 0.0625
        lens = np.array(lens, dtype=np.int64)
        per = np.array(per, dtype=np.int64)
        table, pool_pages = generate.page_tables(seed, lens, None)
        pool_bits = generate.kv_pool(seed, lens, table, pool_pages, width)
        tokens = int(per.sum())
        q_bits = generate.queries(seed, tokens, heads, width)
        seq_id = np.repeat(np.arange(len(lens)), per).astype(np.int32)
        q_pos = np.concatenate([lens[b] - per[b] + np.arange(per[b])
                                for b in range(len(lens))]).astype(np.int32)
        rng = np.random.default_rng(seed)
        idx = np.full((tokens, k), -1, np.int32)
        k_len = np.zeros(tokens, np.int32)
        masks = []
        for t in range(tokens):
            kl_seq = int(lens[seq_id[t]])
            vis = min(kl_seq, int(q_pos[t]) + 1)
            n = min(vis, k - 6)
            sel = rng.choice(vis, size=n, replace=False)
            junk = [-1, int(q_pos[t]) + 1, kl_seq, 2 ** 31 - 1, -2, -2 ** 31]
            row = np.concatenate([sel, junk]).astype(np.int64)
            rng.shuffle(row)
            kl = min(k, len(row))
            idx[t, :kl] = row[:kl]
            k_len[t] = kl
            idx[t, kl:] = rng.integers(0, max(1, vis), size=k - kl)  # stale padding
            v = idx[t, : k_len[t]].astype(np.int64)
            v = v[(v >= 0) & (v <= q_pos[t]) & (v < kl_seq)]
            m = np.zeros(kl_seq, dtype=bool)
            m[v] = True
            masks.append(m)
        rows = generate.bf16_to_f64(pool_bits)
        q = generate.bf16_to_f64(q_bits)
        w_uk = np.broadcast_to(np.eye(width), (heads, width, width)).copy()
        w_uv = np.broadcast_to(np.eye(512, width), (heads, 512, width)).copy()
        exp_out = np.zeros((tokens, heads, 512))
        exp_lse = np.zeros((tokens, heads))
        for t in range(tokens):
            b = int(seq_id[t])
            pos = np.arange(lens[b])
            latent = rows[table[b, pos // 64].astype(np.int64) * 64 + pos % 64]
            res = mla_attention.mla_attention_core(q[t : t + 1], latent, w_uk, w_uv,
                                                   masks[t][None, :], scale=scale)
            exp_out[t] = res.out[0]
            exp_lse[t] = res.lse[0]
        out[f"{name}__meta"] = np.array([seed, heads, width, pool_pages])
        out[f"{name}__kv_len"] = lens
        out[f"{name}__per_seq"] = per
        out[f"{name}__page_table"] = table
        out[f"{name}__seq_id"] = seq_id
        out[f"{name}__q_pos"] = q_pos
        out[f"{name}__idx"] = idx
        out[f"{name}__k_len"] = k_len
        out[f"{name}__scale"] = np.array(scale)
        out[f"{name}__q_sha256"] = np.array(hashlib.sha256(q_bits.tobytes()).hexdigest())
        out[f"{name}__pool_sha256"] = np.array(hashlib.sha256(pool_bits.tobytes()).hexdigest())
        out[f"{name}__out"] = exp_out
        out[f"{name}__lse"] = exp_lse
    np.savez_compressed(HERE / "sparse_cases.npz", **out)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <reference checkout>")
    reference = Path(sys.argv[1])
    copy_philox(reference)
    upstream_cases(reference)
    paged_cases(reference)
    sparse_cases(reference)
    print("golden fixtures written to", HERE)
