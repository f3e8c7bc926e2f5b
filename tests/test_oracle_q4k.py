"""Pins the oracle's Q4_K / Q8_K restatement (oracle/hkv_oracle_q4k.c).

Q4_K decoding is compared with gguf.quants.dequantize (the gguf package's
independent implementation of the GGUF block format); the Q8_K quantiser
and the Q4_K x Q8_K dot product, which gguf does not implement, are checked
against their definitions in float64.
"""
from __future__ import annotations

import numpy as np
import pytest

import cpu_oracle as o


def random_q4k_blocks(rng, n_blocks):
    """Random but well-formed Q4_K blocks: every byte random except the two
    f16 super-scales, kept finite and positive like a quantiser's output."""
    b = rng.integers(0, 256, size=(n_blocks, o.Q4K_BYTES), dtype=np.uint8)
    d = rng.uniform(1e-4, 2e-3, n_blocks).astype(np.float16)
    dmin = rng.uniform(1e-4, 2e-3, n_blocks).astype(np.float16)
    b[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
    b[:, 2:4] = dmin.view(np.uint8).reshape(-1, 2)
    return b


def test_q4k_dequant_matches_gguf():
    quants = pytest.importorskip("gguf.quants")
    import gguf
    rng = np.random.default_rng(0)
    rows, cols = 37, 2560
    blocks = random_q4k_blocks(rng, rows * cols // 256).reshape(rows, -1)
    ours = o.q4k_dequant(blocks, cols)
    ref = quants.dequantize(blocks, gguf.GGMLQuantizationType.Q4_K)
    assert ref.shape == (rows, cols)
    assert np.array_equal(ours, ref.astype(np.float32))


def test_q8k_quantize_definition():
    rng = np.random.default_rng(1)
    x = rng.standard_normal(4 * 256).astype(np.float32)
    x[256:512] *= -3.0
    x[512:768] = 0.0                    # an all-zero block
    x[768 + 5] = 7.0                    # ties in magnitude: the first one wins
    x[768 + 9] = -7.0
    q = o.q8k_quantize(x).reshape(4, o.Q8K_BYTES)
    for b in range(4):
        xb = x[256 * b:256 * (b + 1)]
        d = q[b, :4].copy().view(np.float32)[0]
        qs = q[b, 4:260].view(np.int8).astype(np.int32)
        bs = q[b, 260:292].copy().view(np.int16).astype(np.int32)
        if not np.any(xb):
            assert d == 0 and not np.any(qs) and not np.any(bs)
            continue
        j = int(np.argmax(np.abs(xb)))
        assert qs[j] == -127                      # the largest element maps to -127
        iscale = np.float32(-127.0) / xb[j]
        assert d == np.float32(1.0) / iscale
        want = np.minimum(127, np.rint((iscale * xb).astype(np.float32))).astype(np.int32)
        assert np.array_equal(qs, want)
        assert np.array_equal(bs, qs.reshape(16, 16).sum(1))
    assert q[3, 4 + 5].view(np.int8) == -127 and q[3, 4 + 9].view(np.int8) == 127


def test_q4k_q8k_dot_is_the_decoded_dot():
    rng = np.random.default_rng(2)
    nb = 38  # one 9728-wide row
    w = random_q4k_blocks(rng, nb).reshape(-1)
    x = rng.standard_normal(nb * 256).astype(np.float32)
    a = o.q8k_quantize(x)
    wd = o.q4k_dequant(w, nb * 256).reshape(-1).astype(np.float64)
    ad = o.q8k_dequant(a).astype(np.float64)
    exact = float(np.dot(wd, ad))
    got = o.q4k_dot_q8k(w, a)
    scale = float(np.abs(wd * ad).sum())
    assert abs(got - exact) <= 1e-6 * scale, (got, exact)


def test_gemv_rows_are_dots():
    rng = np.random.default_rng(3)
    rows, cols = 64, 2560
    w = random_q4k_blocks(rng, rows * cols // 256).reshape(rows, -1)
    x = rng.standard_normal((2, cols)).astype(np.float32)
    y = o.q4k_gemv(w, rows, cols, x)
    for e in range(2):
        a = o.q8k_quantize(x[e])
        for r in (0, 17, 63):
            assert y[e, r] == np.float32(o.q4k_dot_q8k(w[r], a))


def test_rms_norm_and_silu():
    rng = np.random.default_rng(4)
    x = rng.standard_normal((3, 2560)).astype(np.float32) * 5
    w = rng.standard_normal(2560).astype(np.float32)
    eps = 1e-6
    y = o.rms_norm_mul(x, eps, w)
    xd = x.astype(np.float64)
    ref = xd / np.sqrt((xd * xd).mean(1, keepdims=True) + eps) * w
    assert np.max(np.abs(y - ref)) <= 1e-5 * np.max(np.abs(ref))
    g = rng.standard_normal(9728).astype(np.float32) * 4
    u = rng.standard_normal(9728).astype(np.float32)
    s = o.silu_mul(g, u)
    gd = g.astype(np.float64)
    assert np.allclose(s, gd / (1 + np.exp(-gd)) * u, rtol=1e-6, atol=1e-7)
