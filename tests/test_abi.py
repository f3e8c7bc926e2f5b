"""The C ABI and the engine's host-side bookkeeping, on a host-only engine (CPU).

A host-only engine (device = -1) runs the real slot / page / reservation /
copy-on-write logic of libhkv.so without touching a GPU; its compute calls
fail with HKV_ERR_NO_DEVICE (there is no CPU fallback).  Failure cases are
injected on the host: pool exhaustion, double release, bad slot ids, range
errors -- each must leave no partial state.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]


@pytest.fixture
def eng(hkv_lib):
    import hkv
    e = hkv.Engine(n_layers=2, n_pages=64, max_slots=8, context_length=4096, device=-1,
                   lib=hkv_lib)
    yield e
    e.close()


def test_exports_every_declared_symbol(hkv_lib):
    import hkv
    declared = set()
    for header in (REPO / "include").glob("*.h"):
        declared |= set(hkv.header_functions(header))
    assert len(declared) >= 25
    for name in declared:
        assert hasattr(hkv_lib, name), name
    assert declared == set(hkv.SIGNATURES), declared ^ set(hkv.SIGNATURES)
    assert hkv_lib.hkv_abi_version() == 3


def test_config_default_is_the_backbone_shape(hkv_lib):
    import hkv
    cfg = hkv.Config()
    assert hkv_lib.hkv_config_default(cfg) == 0
    assert (cfg.n_layers, cfg.n_head, cfg.n_head_kv, cfg.head_dim, cfg.page_tokens,
            cfg.context_length) == (36, 32, 8, 128, 16, 32768)
    assert cfg.rope_freq_base == pytest.approx(1e6)


def test_create_rejects_unsupported_shapes(hkv_lib):
    import hkv
    with pytest.raises(hkv.HkvError):
        hkv.Engine(head_dim=64, device=-1, lib=hkv_lib)
    with pytest.raises(hkv.HkvError):
        hkv.Engine(n_head=24, n_head_kv=8, device=-1, lib=hkv_lib)
    with pytest.raises(hkv.HkvError):
        hkv.Engine(page_tokens=32, device=-1, lib=hkv_lib)


def test_engine_rope_tables_match_reference_code(hkv_lib):
    import hashlib
    import hkv
    g = np.load(REPO / "tests" / "golden" / "rope_table_ref.npz")
    e = hkv.Engine(n_layers=1, n_pages=4, max_slots=1, device=-1, lib=hkv_lib)
    cos, sin = e.rope_tables()
    e.close()
    assert hashlib.sha256(cos.tobytes()).digest() == g["cos_sha256"].tobytes()
    assert hashlib.sha256(sin.tobytes()).digest() == g["sin_sha256"].tobytes()


def test_slot_lifecycle_and_scoped_release(eng):
    import hkv
    with eng.acquire_backend_kv_cache_slot(40) as lease:
        s = lease.slot
        assert eng.length(s) == 0
        st = eng.stats()
        assert st["live_slots"] == 1 and st["reserved"] == 3  # ceil(40/16)
    st = eng.stats()
    assert st["live_slots"] == 0 and st["reserved"] == 0 and st["free_pages"] == 64
    with pytest.raises(hkv.HkvError) as ei:
        eng.release(s)
    assert ei.value.status == hkv.HKV_ERR_BAD_SLOT


def test_bad_slot_ids(eng):
    import hkv
    for bad in (-1, 8, 3):
        with pytest.raises(hkv.HkvError) as ei:
            eng.length(bad)
        assert ei.value.status == hkv.HKV_ERR_BAD_SLOT
    assert "not live" in eng.last_error()


def test_compute_calls_fail_without_device(eng):
    import hkv
    s = eng.acquire(16)
    with pytest.raises(hkv.HkvError) as ei:
        eng.rope_append(0, [s], 16, 16)
    assert ei.value.status == hkv.HKV_ERR_NO_DEVICE
    with pytest.raises(hkv.HkvError) as ei:
        eng.decode_attn(0, [s], 16, 16)
    assert ei.value.status == hkv.HKV_ERR_NO_DEVICE
    with pytest.raises(hkv.HkvError) as ei:
        eng.sync_check()
    assert ei.value.status == hkv.HKV_ERR_NO_DEVICE


def test_reservation_exhaustion_leaves_no_state(eng):
    import hkv
    a = eng.acquire(16 * 60)  # reserves 60 of 64 pages
    before = eng.stats()
    with pytest.raises(hkv.HkvError) as ei:
        eng.acquire(16 * 5)
    assert ei.value.status == hkv.HKV_ERR_OOM
    assert eng.stats() == before
    b = eng.acquire(16 * 4)
    assert eng.stats()["reserved"] == 64
    eng.release(a)
    eng.release(b)
    assert eng.stats()["reserved"] == 0


def test_slot_table_exhaustion(eng):
    import hkv
    slots = [eng.acquire(0) for _ in range(8)]
    with pytest.raises(hkv.HkvError) as ei:
        eng.acquire(0)
    assert ei.value.status == hkv.HKV_ERR_OOM
    for s in slots:
        eng.release(s)
    assert eng.stats()["live_slots"] == 0


def test_capacity_and_range_errors(eng):
    import hkv
    with pytest.raises(hkv.HkvRangeError):
        eng.acquire(5000)  # beyond the context length
    s = eng.acquire(0)
    with pytest.raises(IndexError):  # std::out_of_range counterpart
        eng.set_length(s, 5)
    with pytest.raises(hkv.HkvRangeError):
        eng.advance([s], 1)  # no row written yet
    with pytest.raises(hkv.HkvRangeError):
        eng.fork(s, 1)
    eng.release(s)


def test_prefix_errors_and_unpublished_key(eng):
    import hkv
    s = eng.acquire(0)
    with pytest.raises(hkv.HkvRangeError):
        eng.publish(0xABC, 10, s)  # the slot holds 0 tokens
    with pytest.raises(hkv.HkvError) as ei:
        eng.drop(0xABC, 10)
    assert ei.value.status == hkv.HKV_ERR_NOT_FOUND
    # an unpublished key acquires an empty slot
    t = eng.acquire(32, share=(0xABC, 10))
    assert eng.length(t) == 0
    eng.release(s)
    eng.release(t)


def test_header_documents_reference_sites():
    text = (REPO / "include" / "hkv.h").read_text()
    for site in (":1191-1208", ":1210-1220", ":5748-5749", ":5750-5786", ":489-506"):
        assert site in text
