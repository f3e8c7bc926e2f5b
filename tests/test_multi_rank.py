"""Multi-rank host logic on CPU: gloo process groups of world size 2.

* KV-head split of one long request: each rank runs the oracle on its share
  of KV heads (what its engine holds) and the all-gather reassembles the
  head-major output -- it must equal the single-rank result bit for bit.
* Slot sharding: every request lands on exactly one rank.
* Failure detection: a rank that never joins makes the others fail with a
  timeout instead of hanging.
"""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup(rank, world, port, timeout_s=60):
    import datetime
    import torch.distributed as dist
    for p in (str(REPO / "higgs-audio.cpp_b200"), str(REPO / "oracle")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _head_split_worker(rank, world, port):
    import torch
    dist = _setup(rank, world, port)
    import cpu_oracle
    import synth
    from hkv_dist import HeadSplit
    import hkv

    split = HeadSplit(world=world, rank=rank)
    # the rank's engine shape is valid for the library
    eng = hkv.Engine(n_layers=2, n_pages=8, max_slots=2, device=-1, **split.engine_shape())
    eng.close()
    lens = [37, 300]
    q = synth.normal(1, (2, 32, 128))
    ks = [cpu_oracle.f32_to_f16(synth.normal(10 + i, (L, 8, 128))) for i, L in enumerate(lens)]
    vs = [cpu_oracle.f32_to_f16(synth.normal(20 + i, (L, 8, 128))) for i, L in enumerate(lens)]
    full = cpu_oracle.decode_attn(q, ks, vs)
    local = cpu_oracle.decode_attn(split.slice_q(q), [split.slice_kv(k) for k in ks],
                                   [split.slice_kv(v) for v in vs])
    assert local.shape == (2, split.local_q_heads * 128)
    gathered = split.gather_output(torch.from_numpy(local)).numpy()
    assert np.array_equal(gathered, full)
    dist.destroy_process_group()


def _shard_worker(rank, world, port):
    dist = _setup(rank, world, port)
    from hkv_dist import shard_requests
    mine = shard_requests(range(11), world, rank)
    everyone = [None] * world
    dist.all_gather_object(everyone, mine)
    flat = sorted(r for part in everyone for r in part)
    assert flat == list(range(11))
    assert all(len(set(a) & set(b)) == 0 for i, a in enumerate(everyone)
               for b in everyone[i + 1:])
    dist.destroy_process_group()


def _lonely_worker(rank, world, port):
    import time
    if rank == 1:
        return  # never joins
    t0 = time.time()
    try:
        _setup(rank, world, port, timeout_s=3)
    except Exception as e:  # DistStoreError / RuntimeError on timeout
        assert time.time() - t0 < 60
        assert "timeout" in str(e).lower() or "timed out" in str(e).lower(), str(e)
        return
    raise AssertionError("init_process_group returned without the second rank")


def _spawn(fn, world=2):
    import torch.multiprocessing as mp
    mp.start_processes(fn, args=(world, _free_port()), nprocs=world, start_method="spawn",
                       join=True)


def test_head_split_allgather_reassembles_heads(hkv_lib):
    _spawn(_head_split_worker)


def test_slot_sharding_places_each_request_once():
    _spawn(_shard_worker)


def test_rank_that_never_joins_times_out():
    _spawn(_lonely_worker)


def test_head_split_shapes():
    sys.path.insert(0, str(REPO / "higgs-audio.cpp_b200"))
    from hkv_dist import HeadSplit
    for world in (1, 2, 4, 8):
        for rank in range(world):
            s = HeadSplit(world=world, rank=rank)
            assert s.local_kv_heads * world == 8
            assert list(s.q_range) == list(range(rank * 32 // world, (rank + 1) * 32 // world))
            assert all(h // 4 in s.kv_range for h in s.q_range)
    with pytest.raises(ValueError):
        HeadSplit(world=3, rank=0)
