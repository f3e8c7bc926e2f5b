"""hkv_decode_attn_noalloc on the GPU: attention without any device allocation.

Some callers cannot call cudaMalloc -- code that has to keep every tensor in
another framework's device pool (the pipeline's ggml backend buffers) or that
runs where an allocation could stall or fail.  They hand this entry point
memory they already own: a page pool in the engine's documented layout, the
RoPE tables, q and out; its own working memory is a fixed static array.

Here the engine fills its cache as usual, the same rows (read back through
hkv_gather, and checked bit for bit against the oracle's own append) are laid
into a caller-owned pool on different physical pages, and two calls in a row
of the new entry point must match both the engine's hkv_decode_attn and the
oracle (exact and ggml_f16 modes) within the parity tolerance, with
hkv_decode_attn_noalloc_sync_check reporting no device-side error after each.
This file is collected last on purpose (a failure here comes after every other
test has run).
"""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DEV = "cuda:0"
TOL = 2e-3  # the same attention tolerance as the other parity tests
G, H, D, L = 8, 32, 128, 2


def rel_err(a, b):
    a = np.asarray(a, np.float64).reshape(-1, D)
    b = np.asarray(b, np.float64).reshape(-1, D)
    return float(np.max(np.abs(a - b).max(1) / np.maximum(np.abs(b).max(1), 1e-30)))


def caller_pool(rows_by_slot, layer, n_layers):
    """Lays logical F16 rows ([R][G][D] uint16 per slot) into a fresh pool in
    the engine's page layout, on pages handed out in reverse order."""
    n_pages = sum((r.shape[0] + 15) // 16 for r, _ in rows_by_slot)
    pool = np.zeros(n_pages * n_layers * 2 * G * 16 * D, np.uint16)
    next_page = n_pages - 1
    page_lists = []
    for k_rows, v_rows in rows_by_slot:
        R = k_rows.shape[0]
        pages = list(range(next_page, next_page - (R + 15) // 16, -1))
        next_page -= len(pages)
        page_lists.append(pages)
        t = np.arange(R)
        page = np.array(pages)[t // 16]
        r = t % 16
        for kv, rows in ((0, k_rows), (1, v_rows)):
            block = ((layer * n_pages + page[:, None]) * 2 + kv) * G + np.arange(G)[None, :]
            chunk = np.arange(16)[None, None, :] ^ (r[:, None, None] & 7)
            base = (block[:, :, None] * (16 * D) + r[:, None, None] * D + chunk * 8)
            idx = base[..., None] + np.arange(8)
            pool[idx.reshape(-1)] = rows.reshape(R, G, 16, 8).reshape(-1)
    return torch.from_numpy(pool.view(np.int16)).to(DEV), page_lists


def test_noalloc_matches_engine_and_oracle_on_two_calls(hkv_lib, oracle, rope_tables):
    import hkv
    import synth

    cos_t, sin_t = rope_tables
    eng = hkv.Engine(n_layers=L, n_pages=256, max_slots=4, device=0, shuffle_seed=99,
                     lib=hkv_lib)
    stream = torch.cuda.current_stream().cuda_stream
    lens = [37, 300, 1000]
    slots = [eng.acquire(n + 1) for n in lens]
    layer = 1
    expect = []  # the oracle's rows of `layer`, [0, n] of each slot
    k_new = synth.normal(7, (3, G, D))
    v_new = synth.normal(8, (3, G, D))
    for i, (s, n) in enumerate(zip(slots, lens)):
        for lay in range(L):
            k = synth.normal(50 + 10 * i + lay, (n, G, D))
            v = synth.normal(80 + 10 * i + lay, (n, G, D))
            eng.rope_append_range(lay, s, n, torch.from_numpy(k).to(DEV),
                                  torch.from_numpy(v).to(DEV), stream)
            if lay == layer:
                k16, v16 = oracle.append_rows(k, v, np.arange(n), cos_t, sin_t)
                kn, vn = oracle.append_rows(k_new[i:i + 1], v_new[i:i + 1], np.array([n]),
                                            cos_t, sin_t)
                expect.append((np.concatenate([k16, kn]), np.concatenate([v16, vn])))
        eng.advance([s], n)
    eng.rope_append(layer, slots, torch.from_numpy(k_new).to(DEV),
                    torch.from_numpy(v_new).to(DEV), stream)

    # the rows the engine now holds, [0, used] of each slot: bit-exact
    rows = []
    for s, n, (ek, ev) in zip(slots, lens, expect):
        kb = torch.empty((n + 1, G, D), dtype=torch.int16, device=DEV)
        vb = torch.empty_like(kb)
        eng.gather(s, layer, 0, n + 1, kb, vb, stream)
        torch.cuda.synchronize()
        rows.append((kb.cpu().numpy().view(np.uint16), vb.cpu().numpy().view(np.uint16)))
        assert np.array_equal(rows[-1][0], ek) and np.array_equal(rows[-1][1], ev)
    pool, page_lists = caller_pool(rows, layer, L)
    cos, sin = eng.rope_tables()
    cos_d = torch.from_numpy(cos).to(DEV)
    sin_d = torch.from_numpy(sin).to(DEV)
    view = hkv.PagedView(pool.data_ptr(), sum(len(p) for p in page_lists), L, G,
                         cos_d.data_ptr(), sin_d.data_ptr(), cos.shape[0])

    calls = [([0, 1, 2], 11), ([2, 0], 12)]  # two calls in a row, different batches
    for order, seed in calls:
        qh = synth.normal(seed, (len(order), H, D))
        q = torch.from_numpy(qh).to(DEV)
        ref = torch.empty((len(order), H * D), device=DEV)
        got = torch.full((len(order), H * D), float("nan"), device=DEV)
        eng.decode_attn(layer, [slots[i] for i in order], q, ref, stream)
        hkv.decode_attn_noalloc(view, layer, [lens[i] for i in order],
                                [page_lists[i] for i in order], q, got, stream, lib=hkv_lib)
        hkv.decode_attn_noalloc_sync_check(stream, lib=hkv_lib)
        g = got.cpu().numpy()
        assert np.all(np.isfinite(g))
        assert rel_err(g, ref.cpu().numpy()) <= TOL, order
        qr = np.stack([oracle.rope_neox(qh[j], cos_t[lens[i]], sin_t[lens[i]])
                       for j, i in enumerate(order)])
        ks = [expect[i][0] for i in order]
        vs = [expect[i][1] for i in order]
        for mode in (oracle.EXACT, oracle.GGML_F16):
            err = rel_err(g, oracle.decode_attn(qr, ks, vs, mode))
            assert err <= TOL, (order, mode, err)
    eng.sync_check(stream)
    eng.close()


def test_noalloc_rejects_batches_beyond_its_scratch(hkv_lib):
    import hkv
    pool = torch.zeros(16 * L * 2 * G * 16 * D, dtype=torch.int16, device=DEV)
    tab = torch.zeros((32768, 64), device=DEV)
    view = hkv.PagedView(pool.data_ptr(), 16, L, G, tab.data_ptr(), tab.data_ptr(), 32768)
    q = torch.zeros((4000, H, D), device=DEV)
    out = torch.zeros((4000, H * D), device=DEV)
    with pytest.raises(hkv.HkvRangeError, match="static scratch"):
        hkv.decode_attn_noalloc(view, 0, [0] * 4000, [[0]] * 4000, q, out, lib=hkv_lib)
    with pytest.raises(hkv.HkvRangeError, match="outside the pool"):
        hkv.decode_attn_noalloc(view, 0, [20], [[0, 16]], q, out, lib=hkv_lib)
    with pytest.raises(hkv.HkvRangeError, match="position"):
        hkv.decode_attn_noalloc(view, 0, [40000], [[0]], q, out, lib=hkv_lib)
    torch.cuda.synchronize()
