"""KV-head split of one batch across 2 GPUs with the in-kernel exchange.

Each rank's engine holds 4 of the 8 KV heads; hkv_split_step writes every
finished head slice into both ranks' exchange regions over NVLink and
hkv_split_wait waits (bounded) for the layer's slices from both.  Each rank
then checks its full head-major output against the oracle over all 8 KV
heads (2e-3, the parity tolerance) and its caches bit for bit.

Needs two GPUs (skipped otherwise); the ranks are separate processes on
separate GPUs, so the peer waits always have their writer running.
"""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]
TOL = 2e-3
G, H, D = 8, 32, 128


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _DeviceArray:
    """A raw device pointer as a torch tensor view (__cuda_array_interface__)."""

    def __init__(self, ptr, shape):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": "<f4", "data": (ptr, False),
                                         "version": 3, "strides": None}


def _rel_err(a, b):
    a = np.asarray(a, np.float64).reshape(-1, D)
    b = np.asarray(b, np.float64).reshape(-1, D)
    return float(np.max(np.abs(a - b).max(1) / np.maximum(np.abs(b).max(1), 1e-30)))


def _worker(rank, world, port):
    import datetime

    import torch.distributed as dist
    for p in (str(REPO / "higgs-audio.cpp_b200"), str(REPO / "oracle")):
        sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    import cpu_oracle
    import hkv
    import synth
    from hkv_dist import HeadSplit

    dev = f"cuda:{rank}"
    split = HeadSplit(world=world, rank=rank)
    eng = hkv.Engine(n_layers=2, n_pages=256, max_slots=4, device=rank, shuffle_seed=rank + 7,
                     **split.engine_shape())
    stream = torch.cuda.current_stream().cuda_stream
    cos, sin = cpu_oracle.rope_table()
    lens = [700, 37]
    slots = [eng.acquire(L + 4) for L in lens]
    caches = {}
    for e, L in enumerate(lens):
        for layer in range(2):
            k = synth.normal(100 * e + layer, (L, G, D))  # identical on every rank
            v = synth.normal(100 * e + layer + 50, (L, G, D))
            eng.rope_append_range(layer, slots[e], L, torch.from_numpy(split.slice_kv(k)).to(dev),
                                  torch.from_numpy(split.slice_kv(v)).to(dev), stream)
            caches[(e, layer)] = list(cpu_oracle.append_rows(k, v, np.arange(L), cos, sin))
        eng.advance([slots[e]], L)
    handles = [None] * world
    dist.all_gather_object(handles, eng.split_export(world, rank))
    eng.split_connect(handles)
    dist.barrier()
    outs = []
    for layer in range(2):
        out_ptr, row_floats = eng.split_output(layer)
        assert row_floats == H * D
        outs.append(torch.as_tensor(_DeviceArray(out_ptr, (4, row_floats)), device=dev))
    worst = 0.0
    for step in range(3):
        pos = np.array([eng.length(s) for s in slots])
        for layer in range(2):
            q = synth.normal(1000 * step + layer, (2, H, D))
            k = synth.normal(1000 * step + layer + 10, (2, G, D))
            v = synth.normal(1000 * step + layer + 20, (2, G, D))
            eng.split_step(layer, slots, torch.from_numpy(split.slice_q(q)).to(dev),
                           torch.from_numpy(split.slice_kv(k)).to(dev),
                           torch.from_numpy(split.slice_kv(v)).to(dev), stream)
            eng.split_wait(layer, stream)
            torch.cuda.synchronize()
            got = outs[layer][:2].cpu().numpy().copy()
            k16, v16 = cpu_oracle.append_rows(k, v, pos, cos, sin)
            ks, vs, qr = [], [], []
            for e in range(2):
                caches[(e, layer)][0] = np.concatenate([caches[(e, layer)][0], k16[e:e + 1]])
                caches[(e, layer)][1] = np.concatenate([caches[(e, layer)][1], v16[e:e + 1]])
                ks.append(caches[(e, layer)][0])
                vs.append(caches[(e, layer)][1])
                qr.append(cpu_oracle.rope_neox(q[e], cos[pos[e]], sin[pos[e]]))
            ref = cpu_oracle.decode_attn(np.stack(qr), ks, vs)
            err = _rel_err(got, ref)
            worst = max(worst, err)
            assert err <= TOL, (rank, step, layer, err)
        eng.advance(slots, 1)
    # this rank's caches hold its own KV heads, bit for bit
    for e, s in enumerate(slots):
        n = eng.length(s)
        kb = torch.empty((n, split.local_kv_heads, D), dtype=torch.int16, device=dev)
        vb = torch.empty_like(kb)
        eng.gather(s, 1, 0, n, kb, vb, stream)
        torch.cuda.synchronize()
        assert np.array_equal(kb.cpu().numpy().view(np.uint16), split.slice_kv(caches[(e, 1)][0]))
        assert np.array_equal(vb.cpu().numpy().view(np.uint16), split.slice_kv(caches[(e, 1)][1]))
    eng.sync_check(stream)
    dist.barrier()
    eng.split_disconnect()  # close the peers' mappings before anyone frees a region
    dist.barrier()
    eng.close()
    dist.destroy_process_group()


def test_split_exchange_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    mp.start_processes(_worker, args=(2, _free_port()), nprocs=2, start_method="spawn", join=True)


def _silent_peer_worker(rank, world, port):
    """Rank 1 connects but never runs its step: rank 0's bounded arrival wait
    must give up (HKV_ERR_TIMEOUT at hkv_sync_check) and leave the engine
    usable.  Nobody dies or faults; rank 1 only stays away between steps."""
    import datetime

    import torch.distributed as dist
    for p in (str(REPO / "higgs-audio.cpp_b200"), str(REPO / "oracle")):
        sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    import hkv
    from hkv_dist import HeadSplit

    dev = f"cuda:{rank}"
    split = HeadSplit(world=world, rank=rank)
    eng = hkv.Engine(n_layers=1, n_pages=16, max_slots=2, device=rank, **split.engine_shape())
    stream = torch.cuda.current_stream().cuda_stream
    s = eng.acquire(40)
    kv = torch.randn((20, split.local_kv_heads, D), device=dev)
    eng.rope_append_range(0, s, 20, kv, kv, stream)
    eng.advance([s], 20)
    handles = [None] * world
    dist.all_gather_object(handles, eng.split_export(world, rank))
    eng.split_connect(handles)
    dist.barrier()
    if rank == 0:
        q = torch.randn((1, split.local_q_heads, D), device=dev)
        k = torch.randn((1, split.local_kv_heads, D), device=dev)
        eng.split_step(0, [s], q, k, k, stream)
        eng.split_wait(0, stream)  # rank 1 never sends its slices
        with pytest.raises(hkv.HkvError) as ei:
            eng.sync_check(stream)
        assert ei.value.status == hkv.HKV_ERR_TIMEOUT, ei.value
        # the context is still good: an ordinary call works and reports clean
        out = torch.empty((1, split.local_q_heads * D), device=dev)
        eng.decode_attn(0, [s], q, out, stream)
        eng.sync_check(stream)
        assert torch.isfinite(out).all()
    dist.barrier()
    eng.split_disconnect()
    dist.barrier()
    eng.close()
    dist.destroy_process_group()


def test_split_wait_times_out_without_peer():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    mp.start_processes(_silent_peer_worker, args=(2, _free_port()), nprocs=2,
                       start_method="spawn", join=True)
