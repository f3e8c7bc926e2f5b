"""The oracle against the reference's known answers and golden fixtures (CPU).

Before the oracle is trusted as the reference for the GPU path it is pinned here:
  * its BF16 RoPE table against the reference's own table code (fixture made
    by compiling make_bf16_rope_table from the reference source);
  * its F16 conversion against numpy's float16 (round to nearest even);
  * its append against the known-answer pattern of
    self_check_backend_kv_cache_write (src/higgs_pipeline.cpp:6960-6986);
  * its RoPE against an independent numpy restatement with each F32 op
    rounded separately (:489-506);
  * its attention against an independent float64 numpy restatement of the
    reference graph (materialised GQA repeat, QK, scale, softmax, PV,
    :5750-5786) and the timed graph restatement.
"""
from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"


def rel_err(a, b):
    """Max over heads of max|a-b| / max|b| within the head: the tolerance metric."""
    a = np.asarray(a, np.float64).reshape(-1, 128)
    b = np.asarray(b, np.float64).reshape(-1, 128)
    return float(np.max(np.abs(a - b).max(1) / np.maximum(np.abs(b).max(1), 1e-30)))


def rope_numpy(x, c, s):
    """NEOX RoPE with every F32 product and sum rounded separately."""
    half = x.shape[-1] // 2
    x0, x1 = x[..., :half], x[..., half:]
    a = (x0 * c).astype(np.float32)
    b = (x1 * s).astype(np.float32)
    d = (x0 * s).astype(np.float32)
    e = (x1 * c).astype(np.float32)
    return np.concatenate([(a - b).astype(np.float32), (d + e).astype(np.float32)], -1)


def attn_graph_f64(q, k_cache, v_cache, rep=4):
    """float64 numpy restatement of the reference graph for one slot."""
    k = k_cache.astype(np.float64)
    v = v_cache.astype(np.float64)
    k4 = np.repeat(k, rep, axis=1)  # head h -> kv head h // rep
    v4 = np.repeat(v, rep, axis=1)
    scale = float(np.float32(1) / np.sqrt(np.float32(128)))
    kq = np.einsum("jhd,hd->hj", k4, q.astype(np.float64)) * scale
    kq = np.exp(kq - kq.max(1, keepdims=True))
    kq /= kq.sum(1, keepdims=True)
    return np.einsum("hj,jhd->hd", kq, v4).reshape(-1)


def test_rope_table_matches_reference_code(oracle, rope_tables):
    g = np.load(GOLDEN / "rope_table_ref.npz")
    cos, sin = rope_tables
    rows = g["rows"]
    assert np.array_equal(cos[rows].view(np.uint32), g["cos_rows"].view(np.uint32))
    assert np.array_equal(sin[rows].view(np.uint32), g["sin_rows"].view(np.uint32))
    assert hashlib.sha256(cos.tobytes()).digest() == g["cos_sha256"].tobytes()
    assert hashlib.sha256(sin.tobytes()).digest() == g["sin_sha256"].tobytes()


def test_rope_table_properties(rope_tables):
    cos, sin = rope_tables
    assert cos.shape == (32768, 64)
    assert np.all(cos[0] == 1.0) and np.all(sin[0] == 0.0)
    # every entry is a BF16 value stored as F32
    assert np.all((cos.view(np.uint32) & 0xFFFF) == 0)
    assert np.all((sin.view(np.uint32) & 0xFFFF) == 0)
    assert np.all(np.abs(cos) <= 1.0) and np.all(np.abs(sin) <= 1.0)


def test_bf16_round_ties_to_even(oracle):
    # 1 + 2^-8 is exactly halfway between 1 and 1 + 2^-7: ties to even -> 1.
    assert oracle.bf16_round(1.0 + 2.0 ** -8) == 1.0
    assert oracle.bf16_round(1.0 + 3 * 2.0 ** -8) == 1.0 + 2.0 ** -6
    assert oracle.bf16_round(-0.0) == 0.0 and np.signbit(oracle.bf16_round(-0.0))


def test_f16_conversion_matches_numpy(oracle):
    rng = np.random.default_rng(0)
    bits = rng.integers(0, 2 ** 32, size=2_000_000, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32)
    x = x[np.isfinite(x)]
    edge = np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, 65536.0, 2.0 ** -24, 2.0 ** -25,
                     3 * 2.0 ** -26, 2.0 ** -14, 2.0 ** -14 - 2.0 ** -25, 1.0 + 2.0 ** -11,
                     1.0 + 3 * 2.0 ** -11, -1.5, 1e-8, 1e8], np.float32)
    x = np.concatenate([x, edge, rng.standard_normal(1_000_000).astype(np.float32)])
    ours = oracle.f32_to_f16(x)
    with np.errstate(over="ignore"):
        ref = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(ours, ref)
    back = oracle.f16_to_f32(ref)
    assert np.array_equal(back.view(np.uint32),
                          ref.view(np.float16).astype(np.float32).view(np.uint32))


def test_append_selfcheck_known_answer(oracle, rope_tables):
    g = np.load(GOLDEN / "append_selfcheck.npz")
    cos, sin = rope_tables
    k16, v16 = oracle.append_rows(g["k"][None], g["v"][None], np.array([int(g["pos"])]),
                                  cos, sin, rope=False)
    assert np.array_equal(k16[0], g["k_f16"])
    assert np.array_equal(v16[0], g["v_f16"])
    # and the values read back are the written ones, as the reference requires
    assert np.array_equal(oracle.f16_to_f32(k16[0]), g["k"])
    assert np.array_equal(oracle.f16_to_f32(v16[0]), g["v"])


def test_layout_selfcheck_known_answer():
    g = np.load(GOLDEN / "layout_selfcheck.npz")
    L, G, D, cap = (int(g[k]) for k in ("layers", "kv_heads", "head_dim", "capacity"))

    def offset(layer, pos, head, dim):  # ((layer*cap + pos)*kvh + head)*hd + dim
        return ((layer * cap + pos) * G + head) * D + dim

    assert offset(0, 0, 0, 0) == int(g["front"])
    assert offset(*[int(c) for c in g["back_coord"]]) == int(g["back"])
    # per-layer logical rows are [pos][head][dim], the order hkv_gather returns
    assert offset(1, 0, 0, 0) - offset(0, 0, 0, 0) == cap * G * D


def test_rope_neox_separately_rounded(oracle, rope_tables):
    import synth
    cos, sin = rope_tables
    x = synth.normal(7, (32, 128))
    for pos in (0, 1, 513, 4097, 32767):
        ours = oracle.rope_neox(x, cos[pos], sin[pos])
        ref = rope_numpy(x, cos[pos], sin[pos])
        assert np.array_equal(ours.view(np.uint32), ref.view(np.uint32)), pos


def test_decode_seed_fixture(oracle, rope_tables):
    g = np.load(GOLDEN / "decode_seed.npz")
    cos, sin = rope_tables
    pos = int(g["pos"])
    k16p, v16p = oracle.append_rows(g["past_k"], g["past_v"], np.arange(pos), cos, sin, rope=False)
    k16n, v16n = oracle.append_rows(g["new_k"], g["new_v"], np.array([pos]), cos, sin, rope=True)
    k_cache = np.concatenate([k16p, k16n])
    v_cache = np.concatenate([v16p, v16n])
    assert np.array_equal(k_cache, g["k_cache"]) and np.array_equal(v_cache, g["v_cache"])
    q = oracle.rope_neox(g["q"][0], cos[pos], sin[pos])[None]
    out = oracle.decode_attn(q, [k_cache], [v_cache])
    assert np.array_equal(out, g["out"])
    ref = attn_graph_f64(q[0], oracle.f16_to_f32(k_cache), oracle.f16_to_f32(v_cache))
    assert rel_err(out[0], ref) < 1e-6


@pytest.mark.parametrize("L", [1, 15, 16, 17, 33, 700])
def test_attention_modes_agree(oracle, L):
    import synth
    q = synth.normal(1, (2, 32, 128))
    ks = [oracle.f32_to_f16(synth.normal(2 + i, (L + i, 8, 128))) for i in range(2)]
    vs = [oracle.f32_to_f16(synth.normal(9 + i, (L + i, 8, 128))) for i in range(2)]
    exact = oracle.decode_attn(q, ks, vs, oracle.EXACT)
    ggml = oracle.decode_attn(q, ks, vs, oracle.GGML_F16)
    for e in range(2):
        ref = attn_graph_f64(q[e], oracle.f16_to_f32(ks[e]), oracle.f16_to_f32(vs[e]))
        assert rel_err(exact[e], ref) < 1e-6
        assert rel_err(ggml[e], ref) < 5e-3  # F16 rounding of q and p


def test_graph_baseline_matches_exact(oracle, rope_tables):
    """The timed F32 graph restatement (F32 cache, materialised repeat)
    agrees with the float64 restatement on the same rows."""
    import synth
    cos, sin = rope_tables
    n, cap = 3, 96
    past = np.array([5, 40, 95], np.int32)
    base = oracle.GraphBaseline(n, cap, cos=cos, sin=sin)
    base.k_cache[:] = synth.normal(3, (n * cap, 8, 128))
    base.v_cache[:] = synth.normal(4, (n * cap, 8, 128))
    q = synth.normal(5, (n, 32, 128))
    k = synth.normal(6, (n, 8, 128))
    v = synth.normal(7, (n, 8, 128))
    out = base.decode_layer(q, k, v, past).copy()
    for e in range(n):
        p = int(past[e])
        rows_k = base.k_cache[e * cap: e * cap + p + 1]
        rows_v = base.v_cache[e * cap: e * cap + p + 1]
        assert np.array_equal(rows_k[p], rope_numpy(k[e], cos[p], sin[p]))
        qr = rope_numpy(q[e], cos[p], sin[p])
        ref = attn_graph_f64(qr, rows_k, rows_v)
        assert rel_err(out[e], ref) < 1e-5
