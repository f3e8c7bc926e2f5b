"""GPU parity: the CUDA path through the C ABI against the CPU oracle.

Contract (tolerances written here, applied to every case):
  * cache contents after append and page-table gathers: BIT-EXACT against the
    oracle's F32->F16 round-to-nearest-even of the roped k / raw v;
  * attention outputs: max relative error <= TOL = 2e-3 against the oracle in
    both modes ("exact" and "ggml_f16"), where the relative error is taken
    per (slot, query head) as max|gpu - ref| / max|ref| over the 128 dims.
Inputs are seeded (repo-owned splitmix64 + Box-Muller), identical for the
GPU and the oracle.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
DEV = "cuda:0"
TOL = 2e-3
G, H, D = 8, 32, 128


def rel_err(a, b):
    a = np.asarray(a, np.float64).reshape(-1, D)
    b = np.asarray(b, np.float64).reshape(-1, D)
    return float(np.max(np.abs(a - b).max(1) / np.maximum(np.abs(b).max(1), 1e-30)))


def to_dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


class Harness:
    """An engine plus the oracle's logical caches of every live slot."""

    def __init__(self, oracle, rope_tables, hkv_lib, n_layers=2, n_pages=1024, max_slots=64,
                 shuffle_seed=12345):
        import hkv
        self.o = oracle
        self.cos, self.sin = rope_tables
        self.n_layers = n_layers
        self.eng = hkv.Engine(n_layers=n_layers, n_pages=n_pages, max_slots=max_slots,
                              device=0, shuffle_seed=shuffle_seed, lib=hkv_lib)
        self.k = {}  # slot -> [layer] -> list of uint16 [n][G][D] row blocks
        self.v = {}
        self.stream = torch.cuda.current_stream().cuda_stream

    def close(self):
        self.eng.sync_check(self.stream)
        self.eng.close()

    def logical(self, slot, layer):
        return (np.concatenate(self.k[slot][layer], 0), np.concatenate(self.v[slot][layer], 0))

    def new_slot(self, capacity=0, share=None, parent=None):
        s = self.eng.acquire(capacity, share)
        if parent is not None:
            n = self.eng.length(s)
            self.k[s] = [[self.logical(parent, l)[0][:n]] for l in range(self.n_layers)]
            self.v[s] = [[self.logical(parent, l)[1][:n]] for l in range(self.n_layers)]
        else:
            self.k[s] = [[np.zeros((0, G, D), np.uint16)] for _ in range(self.n_layers)]
            self.v[s] = [[np.zeros((0, G, D), np.uint16)] for _ in range(self.n_layers)]
        return s

    def fork(self, src, n):
        d = self.eng.fork(src, n)
        self.k[d] = [[self.logical(src, l)[0][:n]] for l in range(self.n_layers)]
        self.v[d] = [[self.logical(src, l)[1][:n]] for l in range(self.n_layers)]
        return d

    def release(self, s):
        self.eng.release(s)
        del self.k[s], self.v[s]

    def prefill(self, slot, T, seed):
        import synth
        pos0 = self.eng.length(slot)
        for layer in range(self.n_layers):
            k = synth.normal(seed * 1000 + layer, (T, G, D))
            v = synth.normal(seed * 1000 + 500 + layer, (T, G, D))
            self.eng.rope_append_range(layer, slot, T, to_dev(k), to_dev(v), self.stream)
            k16, v16 = self.o.append_rows(k, v, np.arange(pos0, pos0 + T), self.cos, self.sin)
            self.k[slot][layer].append(k16)
            self.v[slot][layer].append(v16)
        self.eng.advance([slot], T)

    def decode(self, slots, seed, fused=False):
        """One decode step for `slots` over all layers; returns per-layer
        (gpu_out, exact_ref, ggml_ref)."""
        import synth
        n = len(slots)
        pos = np.array([self.eng.length(s) for s in slots])
        results = []
        for layer in range(self.n_layers):
            q = synth.normal(seed * 7919 + layer, (n, H, D))
            k = synth.normal(seed * 7919 + 100 + layer, (n, G, D))
            v = synth.normal(seed * 7919 + 200 + layer, (n, G, D))
            out = torch.empty((n, H * D), dtype=torch.float32, device=DEV)
            if fused:
                self.eng.decode_step(layer, slots, to_dev(q), to_dev(k), to_dev(v), out,
                                     self.stream)
            else:
                self.eng.rope_append(layer, slots, to_dev(k), to_dev(v), self.stream)
                self.eng.decode_attn(layer, slots, to_dev(q), out, self.stream)
            k16, v16 = self.o.append_rows(k, v, pos, self.cos, self.sin)
            qr = np.stack([self.o.rope_neox(q[e], self.cos[pos[e]], self.sin[pos[e]])
                           for e in range(n)])
            ks, vs = [], []
            for e, s in enumerate(slots):
                self.k[s][layer].append(k16[e:e + 1])
                self.v[s][layer].append(v16[e:e + 1])
                kk, vv = self.logical(s, layer)
                ks.append(kk)
                vs.append(vv)
            exact = self.o.decode_attn(qr, ks, vs, self.o.EXACT)
            ggml = self.o.decode_attn(qr, ks, vs, self.o.GGML_F16)
            results.append((out.cpu().numpy(), exact, ggml))
        self.eng.advance(slots, 1)
        return results

    def gather(self, slot, layer, pos0=0, n=None):
        n = self.eng.length(slot) - pos0 if n is None else n
        kb = torch.empty((n, G, D), dtype=torch.int16, device=DEV)
        vb = torch.empty_like(kb)
        self.eng.gather(slot, layer, pos0, n, kb, vb, self.stream)
        torch.cuda.synchronize()
        return kb.cpu().numpy().view(np.uint16), vb.cpu().numpy().view(np.uint16)

    def check_cache(self, slot):
        for layer in range(self.n_layers):
            gk, gv = self.gather(slot, layer)
            rk, rv = self.logical(slot, layer)
            assert np.array_equal(gk, rk), (slot, layer)
            assert np.array_equal(gv, rv), (slot, layer)


@pytest.fixture
def harness(oracle, rope_tables, hkv_lib):
    made = []

    def make(**kw):
        h = Harness(oracle, rope_tables, hkv_lib, **kw)
        made.append(h)
        return h

    yield make
    for h in made:
        h.close()


def check_outputs(results):
    worst = 0.0
    for out, exact, ggml in results:
        assert np.all(np.isfinite(out))
        e1, e2 = rel_err(out, exact), rel_err(out, ggml)
        assert e1 <= TOL, e1
        assert e2 <= TOL, e2
        worst = max(worst, e1)
    return worst


def test_append_selfcheck_known_answer(harness):
    """self_check_backend_kv_cache_write (:6960-6986): a raw row written at
    layer 0, position 1 reads back unchanged."""
    g = np.load(GOLDEN / "append_selfcheck.npz")
    h = harness(n_layers=2)
    s = h.new_slot(4)
    zero = np.zeros((1, G, D), np.float32)
    h.eng.append(0, [s], to_dev(zero), to_dev(zero), h.stream)
    h.eng.append(1, [s], to_dev(zero), to_dev(zero), h.stream)
    h.eng.advance([s], 1)
    h.eng.append(0, [s], to_dev(g["k"][None]), to_dev(g["v"][None]), h.stream)
    h.eng.append(1, [s], to_dev(zero), to_dev(zero), h.stream)
    h.eng.advance([s], 1)
    k, v = h.gather(s, 0, 1, 1)
    assert np.array_equal(k[0], g["k_f16"]) and np.array_equal(v[0], g["v_f16"])
    k0, _ = h.gather(s, 0, 0, 1)
    assert np.all(k0 == 0)


def test_rope_table_upload_matches_reference(harness, rope_tables):
    import hashlib
    g = np.load(GOLDEN / "rope_table_ref.npz")
    h = harness(n_layers=1, n_pages=8)
    cos, sin = h.eng.rope_tables()
    assert hashlib.sha256(cos.tobytes()).digest() == g["cos_sha256"].tobytes()
    assert hashlib.sha256(sin.tobytes()).digest() == g["sin_sha256"].tobytes()


def test_decode_seed_fixture(harness):
    """Deterministic self-check patterns (:5338-5341, :6996-6998, :6690-6692)."""
    g = np.load(GOLDEN / "decode_seed.npz")
    h = harness(n_layers=1)
    s = h.new_slot(64)
    pos = int(g["pos"])
    for p in range(pos):
        h.eng.append(0, [s], to_dev(g["past_k"][p:p + 1]), to_dev(g["past_v"][p:p + 1]),
                     h.stream)
        h.eng.advance([s], 1)
    out = torch.empty((1, H * D), dtype=torch.float32, device=DEV)
    h.eng.rope_append(0, [s], to_dev(g["new_k"]), to_dev(g["new_v"]), h.stream)
    h.eng.decode_attn(0, [s], to_dev(g["q"]), out, h.stream)
    h.eng.advance([s], 1)
    k, v = h.gather(s, 0)
    assert np.array_equal(k, g["k_cache"]) and np.array_equal(v, g["v_cache"])
    assert rel_err(out.cpu().numpy(), g["out"]) <= TOL


@pytest.mark.parametrize("lengths", [[0], [1, 14, 15, 16], [17, 30, 31, 32, 33],
                                     [255, 256, 257, 1000], [4095]])
def test_ragged_decode(harness, lengths):
    h = harness(n_layers=2, n_pages=1024)
    slots = []
    for i, L in enumerate(lengths):
        s = h.new_slot(L + 4)
        if L:
            h.prefill(s, L, seed=10 + i)
        slots.append(s)
    for step in range(3):
        check_outputs(h.decode(slots, seed=100 + step))
    for s in slots:
        h.check_cache(s)


def test_last_context_position(harness):
    """A slot filled to 32,766 rows decodes its last two positions (32,766 and
    32,767, the final rows of the RoPE table and of the context), next to a
    short slot in the same batch; one more step is refused."""
    import hkv
    h = harness(n_layers=1, n_pages=2048 + 8)
    long_slot = h.new_slot(32768)
    h.prefill(long_slot, 32766, seed=71)
    short = h.new_slot(40)
    h.prefill(short, 21, seed=72)
    for step in range(2):
        check_outputs(h.decode([long_slot, short], seed=400 + step))
    assert h.eng.length(long_slot) == 32768
    with pytest.raises(hkv.HkvRangeError):
        h.decode([long_slot], seed=500)
    k, v = h.gather(long_slot, 0, 32760, 8)
    rk, rv = h.logical(long_slot, 0)
    assert np.array_equal(k, rk[32760:]) and np.array_equal(v, rv[32760:])


def test_config1_single_slot_512_prefill_120_steps(harness):
    """Single slot, one layer: 512 prefilled positions, then 120 steps each
    appending one row and attending a fresh query (the reference's CPU case)."""
    h = harness(n_layers=1, n_pages=64)
    s = h.new_slot(512 + 121)
    h.prefill(s, 512, seed=0)
    worst = 0.0
    for step in range(120):
        worst = max(worst, check_outputs(h.decode([s], seed=1000 + step)))
    h.check_cache(s)
    assert worst <= TOL


@pytest.mark.parametrize("length", [260, 600, 1100, 16000])
def test_single_slot_cluster_merge(harness, length):
    """One slot alone (the batch-1 decode step, one long request): the plan
    gives each KV head a thread-block cluster of 2, 4, 8 or 16 CTAs whose
    partials meet in the first CTA's shared memory (plan_cluster).  Fused and
    separate calls, four steps, against both oracle modes.  At 1,100
    positions (69-72 pages: 8 clusters of 8 CTAs) each attention is one
    launch: no combine launch follows."""
    h = harness(n_layers=1, n_pages=length // 16 + 8)
    s = h.new_slot(length + 8)
    h.prefill(s, length, seed=31)
    torch.cuda.synchronize()
    before = h.eng.stats()["kernel_launches"]
    for step in range(4):
        check_outputs(h.decode([s], seed=600 + step, fused=step % 2 == 0))
    launches = h.eng.stats()["kernel_launches"] - before
    if length == 1100:
        assert launches == 2 * 1 + 2 * 2  # fused: 1; separate: append + attention
    h.check_cache(s)


def test_batched_permuted_pages_many_slots(harness):
    """16 slots, contexts drawn in [256, 4096], permuted physical pages."""
    import synth
    h = harness(n_layers=2, n_pages=16 * 260, shuffle_seed=777)
    lens = synth.uniform_int(3, 16, 256, 4096)
    slots = []
    for i, L in enumerate(lens):
        s = h.new_slot(int(L) + 8)
        h.prefill(s, int(L), seed=200 + i)
        slots.append(s)
    pages = [p for s in slots for p in h.eng.pages(s)]
    assert len(set(pages)) == len(pages)
    assert pages != sorted(pages)  # physical order scrambled
    for step in range(2):
        check_outputs(h.decode(slots, seed=300 + step))
    for s in slots[:4]:
        h.check_cache(s)


def test_fused_step_matches_separate_calls(oracle, rope_tables, hkv_lib):
    hs = [Harness(oracle, rope_tables, hkv_lib, n_layers=2, shuffle_seed=5) for _ in range(2)]
    outs = []
    for fused, h in zip((False, True), hs):
        slots = [h.new_slot(700), h.new_slot(40)]
        h.prefill(slots[0], 600, seed=1)
        h.prefill(slots[1], 33, seed=2)
        res = []
        for step in range(2):
            res += h.decode(slots, seed=50 + step, fused=fused)
        check_outputs(res)
        outs.append([r[0] for r in res])
    for a, b in zip(*outs):
        assert np.array_equal(a, b)
    for h in hs:
        h.close()


@pytest.mark.parametrize("prefix", [768, 770])
def test_prefix_sharing_copy_on_write(harness, prefix):
    """Groups share a reference-prompt prefix through published pages; the
    first append into a shared partial page copies it (770 is not page
    aligned, 768 is)."""
    h = harness(n_layers=2, n_pages=512)
    owner = h.new_slot(prefix)
    h.prefill(owner, prefix, seed=9)
    h.eng.publish(0xC0FFEE, prefix, owner)
    members = [h.new_slot(prefix + 8, share=(0xC0FFEE, prefix), parent=owner) for _ in range(3)]
    for m in members:
        assert h.eng.length(m) == prefix
        assert h.eng.pages(m) == h.eng.pages(owner)[: (prefix + 15) // 16]
    before = h.eng.stats()
    assert before["shared_pages"] == (prefix + 15) // 16
    group = [owner] + members
    for step in range(3):
        check_outputs(h.decode(group, seed=60 + step))
    after = h.eng.stats()
    expect_cow = len(group) if prefix % 16 else 0
    assert after["cow_copies"] - before["cow_copies"] == expect_cow
    for s in group:
        h.check_cache(s)
    # the shared full pages are still shared, the tails are private
    tails = [h.eng.pages(s)[prefix // 16:] for s in group]
    assert len({tuple(t) for t in tails}) == len(group)
    h.eng.drop(0xC0FFEE, prefix)
    for s in group:
        h.release(s)
    assert h.eng.stats()["free_pages"] == 512


def test_fork_and_truncate(harness):
    h = harness(n_layers=2, n_pages=256)
    a = h.new_slot(300)
    h.prefill(a, 250, seed=4)
    b = h.fork(a, 100)
    check_outputs(h.decode([a, b], seed=70))
    h.check_cache(a)
    h.check_cache(b)
    # truncate a (window refresh) and rewrite rows
    h.eng.set_length(a, 200)
    for layer in range(2):
        h.k[a][layer] = [h.logical(a, layer)[0][:200]]
        h.v[a][layer] = [h.logical(a, layer)[1][:200]]
    h.prefill(a, 30, seed=5)
    check_outputs(h.decode([a, b], seed=71))
    h.check_cache(a)
    h.check_cache(b)


def test_slot_churn_reuses_pages(harness):
    """Slots finish and are replaced by fresh prefix-only slots; freed pages
    are reused and every step still matches the oracle."""
    import synth
    h = harness(n_layers=1, n_pages=400, max_slots=32)
    owner = h.new_slot(50)
    h.prefill(owner, 50, seed=31)
    h.eng.publish(7, 50, owner)
    live = [h.new_slot(200, share=(7, 50), parent=owner) for _ in range(8)]
    for i, s in enumerate(live):
        h.prefill(s, int(synth.uniform_int(40 + i, 1, 1, 60)[0]), seed=40 + i)
    rng = np.random.default_rng(0)
    reused = 0
    for step in range(12):
        check_outputs(h.decode(live, seed=500 + step))
        for i in range(len(live)):
            if rng.random() < 0.2:
                old_pages = set(h.eng.pages(live[i]))
                h.release(live[i])
                live[i] = h.new_slot(200, share=(7, 50), parent=owner)
                reused += 1
                del old_pages
    assert reused > 0
    for s in live:
        h.check_cache(s)


def test_full_size_property_constant_values(hkv_lib):
    """Full-size check (per-GPU share of the 256-slot scale-out workload:
    32 slots, contexts up to 16384): with every V row of a (slot, KV head)
    equal to one vector, attention returns that vector whatever K is
    (softmax weights sum to one), for every slot, head and layer."""
    import hkv
    import synth
    n_layers, n = 2, 32
    lens = synth.uniform_int(11, n, 2048, 16384)
    pages = int(sum((L + 16) // 16 + 1 for L in lens))
    eng = hkv.Engine(n_layers=n_layers, n_pages=pages, max_slots=n, device=0, shuffle_seed=9,
                     lib=hkv_lib)
    stream = torch.cuda.current_stream().cuda_stream
    slots = [eng.acquire(int(L) + 1) for L in lens]
    gen = torch.Generator(device=DEV)
    gen.manual_seed(0)
    vconst = torch.randn((n, G, D), generator=gen, device=DEV)
    for e, (s, L) in enumerate(zip(slots, lens)):
        L = int(L)
        for layer in range(n_layers):
            k = torch.randn((L, G, D), generator=gen, device=DEV)
            v = vconst[e].expand(L, G, D).contiguous()
            eng.rope_append_range(layer, s, L, k, v, stream)
        eng.advance([s], L)
    for layer in range(n_layers):
        q = torch.randn((n, H, D), generator=gen, device=DEV) * 3
        k = torch.randn((n, G, D), generator=gen, device=DEV)
        out = torch.empty((n, H * D), device=DEV)
        eng.rope_append(layer, slots, k, vconst.contiguous(), stream)
        eng.decode_attn(layer, slots, q, out, stream)
        expect = vconst.half().float().repeat_interleave(4, dim=1).reshape(n, H * D)
        err = rel_err(out.cpu().numpy(), expect.cpu().numpy())
        assert err <= 1e-4, err  # F32 accumulation over up to 16k rows
    eng.sync_check(stream)
    eng.close()


def test_errors_do_not_touch_the_gpu(harness):
    import hkv
    h = harness(n_layers=2, n_pages=4)
    s = h.new_slot(0)
    q = torch.zeros((1, H, D), device=DEV)
    with pytest.raises(hkv.HkvRangeError):
        h.eng.decode_attn(2, [s], q, q)  # layer out of range
    with pytest.raises(hkv.HkvError) as ei:
        h.eng.decode_attn(0, [s, s], q, q)  # duplicate slot
    assert ei.value.status == hkv.HKV_ERR_INVALID
    with pytest.raises(hkv.HkvError) as ei:
        h.eng.decode_attn(0, [s], q.view(-1)[1:], q)  # misaligned pointer
    assert ei.value.status == hkv.HKV_ERR_INVALID
    big = torch.zeros((80, G, D), device=DEV)
    with pytest.raises(hkv.HkvError) as ei:
        h.eng.rope_append_range(0, s, 80, big, big)  # 5 pages > pool of 4
    assert ei.value.status == hkv.HKV_ERR_OOM
    assert h.eng.stats()["free_pages"] == 4 and h.eng.pages(s) == []
    h.eng.sync_check(h.stream)
