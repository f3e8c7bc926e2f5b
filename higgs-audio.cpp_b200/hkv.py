"""ctypes binding of libhkv.so (include/hkv.h) for Python callers and tests.

The binding mirrors the reference's slot API (src/higgs_pipeline.cpp):
``acquire_backend_kv_cache_slot`` (:1191) -> ``Engine.acquire_backend_kv_cache_slot``
returning a ``ScopedBackendKvCacheSlot`` context manager whose exit releases
the slot (:372-403, :1210); engine errors raise ``HkvError`` (a
``RuntimeError``, as the reference throws ``std::runtime_error``), and
position errors raise ``HkvRangeError`` (an ``IndexError``, the reference's
``std::out_of_range`` at :1138-1140).

Compute calls take device pointers (ints, or objects with ``data_ptr()``)
and a CUDA stream handle (int).  There is no CPU fallback: if the library
is missing, loading it raises.
"""
from __future__ import annotations

import ctypes
import os
import re
from pathlib import Path
from typing import Optional, Sequence

import numpy as np

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("HKV_LIB", _PKG / "lib" / "libhkv.so"))

HKV_OK = 0
HKV_ERR_INVALID = 1
HKV_ERR_OOM = 2
HKV_ERR_BAD_SLOT = 3
HKV_ERR_RANGE = 4
HKV_ERR_CUDA = 5
HKV_ERR_TIMEOUT = 6
HKV_ERR_NO_DEVICE = 7
HKV_ERR_NOT_FOUND = 8
HKV_ERR_DEVICE = 9

KERNEL_APPEND = 0
KERNEL_ATTN = 1
KERNEL_COMBINE = 2
KERNEL_GATHER = 3
KERNEL_STEP = 4


class HkvError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class HkvRangeError(HkvError, IndexError):
    pass


class Config(ctypes.Structure):
    _fields_ = [
        ("n_layers", ctypes.c_int32),
        ("n_head", ctypes.c_int32),
        ("n_head_kv", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("page_tokens", ctypes.c_int32),
        ("context_length", ctypes.c_int32),
        ("rope_freq_base", ctypes.c_float),
        ("max_slots", ctypes.c_int32),
        ("n_pages", ctypes.c_int64),
        ("device", ctypes.c_int32),
        ("shuffle_seed", ctypes.c_uint32),
    ]


class PrefixKey(ctypes.Structure):
    _fields_ = [("hash", ctypes.c_uint64), ("n_tokens", ctypes.c_int64)]


class PoolStats(ctypes.Structure):
    _fields_ = [
        ("n_pages", ctypes.c_int64),
        ("free_pages", ctypes.c_int64),
        ("reserved", ctypes.c_int64),
        ("shared_pages", ctypes.c_int64),
        ("live_slots", ctypes.c_int32),
        ("prefixes", ctypes.c_int32),
        ("page_bytes", ctypes.c_int64),
        ("cow_copies", ctypes.c_int64),
        ("kernel_launches", ctypes.c_int64),
    ]


class PagedView(ctypes.Structure):
    """hkv_paged_view: caller-owned device memory in the engine's page layout."""
    _fields_ = [
        ("pool", ctypes.c_void_p),
        ("n_pages", ctypes.c_int64),
        ("n_layers", ctypes.c_int32),
        ("n_head_kv", ctypes.c_int32),
        ("rope_cos", ctypes.c_void_p),
        ("rope_sin", ctypes.c_void_p),
        ("context_length", ctypes.c_int32),
    ]


class Q4kGemvArgs(ctypes.Structure):
    """hkv_q4k_gemv_args."""
    _fields_ = [("w", ctypes.c_void_p), ("w_up", ctypes.c_void_p), ("rows", ctypes.c_int64),
                ("cols", ctypes.c_int64), ("n", ctypes.c_int32), ("x", ctypes.c_void_p),
                ("norm", ctypes.c_void_p), ("eps", ctypes.c_float), ("residual", ctypes.c_void_p),
                ("y", ctypes.c_void_p), ("tensor_cores", ctypes.c_int32)]


class Q4kQkvArgs(ctypes.Structure):
    """hkv_q4k_qkv_args."""
    _fields_ = [("wq", ctypes.c_void_p), ("wk", ctypes.c_void_p), ("wv", ctypes.c_void_p),
                ("n_head", ctypes.c_int32), ("n_head_kv", ctypes.c_int32), ("cols", ctypes.c_int64),
                ("n", ctypes.c_int32), ("x", ctypes.c_void_p), ("norm", ctypes.c_void_p),
                ("eps", ctypes.c_float), ("q_norm", ctypes.c_void_p), ("k_norm", ctypes.c_void_p),
                ("q_out", ctypes.c_void_p), ("k_out", ctypes.c_void_p), ("v_out", ctypes.c_void_p),
                ("tensor_cores", ctypes.c_int32)]


class BackboneLayer(ctypes.Structure):
    """hkv_backbone_layer: one layer's weight pointers."""
    _fields_ = [(name, ctypes.c_void_p) for name in (
        "attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down",
        "attn_norm", "ffn_norm", "attn_q_norm", "attn_k_norm")]


class BackboneWeights(ctypes.Structure):
    """hkv_backbone_weights."""
    _fields_ = [("hidden", ctypes.c_int32), ("ffn", ctypes.c_int32), ("text_vocab", ctypes.c_int64),
                ("n_codebooks", ctypes.c_int32), ("codebook_size", ctypes.c_int32),
                ("rms_eps", ctypes.c_float), ("layers", ctypes.POINTER(BackboneLayer)),
                ("token_embd", ctypes.c_void_p), ("audio_embd", ctypes.c_void_p),
                ("output_norm", ctypes.c_void_p), ("audio_output", ctypes.c_void_p)]


_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_I32P = ctypes.POINTER(ctypes.c_int32)
_I64P = ctypes.POINTER(ctypes.c_int64)

# name -> (argtypes, restype); every function declared in include/hkv.h.
SIGNATURES = {
    "hkv_abi_version": ([], ctypes.c_int),
    "hkv_status_string": ([ctypes.c_int], ctypes.c_char_p),
    "hkv_last_error": ([_P], ctypes.c_char_p),
    "hkv_config_default": ([ctypes.POINTER(Config)], ctypes.c_int),
    "hkv_engine_create": ([ctypes.POINTER(Config), ctypes.POINTER(_P)], ctypes.c_int),
    "hkv_engine_destroy": ([_P], ctypes.c_int),
    "hkv_slot_acquire": ([_P, _I64, ctypes.POINTER(PrefixKey), _I32P], ctypes.c_int),
    "hkv_slot_release": ([_P, _I32], ctypes.c_int),
    "hkv_slot_fork": ([_P, _I32, _I64, _I32P], ctypes.c_int),
    "hkv_slot_len": ([_P, _I32, _I64P], ctypes.c_int),
    "hkv_slot_set_len": ([_P, _I32, _I64], ctypes.c_int),
    "hkv_slot_advance": ([_P, _I32, _I32P, _I64], ctypes.c_int),
    "hkv_prefix_publish": ([_P, ctypes.POINTER(PrefixKey), _I32], ctypes.c_int),
    "hkv_prefix_drop": ([_P, ctypes.POINTER(PrefixKey)], ctypes.c_int),
    "hkv_slot_pages": ([_P, _I32, _I32P, _I64, _I64P], ctypes.c_int),
    "hkv_pool_stats_get": ([_P, ctypes.POINTER(PoolStats)], ctypes.c_int),
    "hkv_append": ([_P, _I32, _I32, _I32P, _P, _P, _P], ctypes.c_int),
    "hkv_rope_append": ([_P, _I32, _I32, _I32P, _P, _P, _P], ctypes.c_int),
    "hkv_rope_append_range": ([_P, _I32, _I32, _I64, _P, _P, _P], ctypes.c_int),
    "hkv_decode_attn": ([_P, _I32, _I32, _I32P, _P, _P, _P], ctypes.c_int),
    "hkv_decode_step": ([_P, _I32, _I32, _I32P, _P, _P, _P, _P, _P], ctypes.c_int),
    "hkv_gather": ([_P, _I32, _I32, _I64, _I64, _P, _P, _P], ctypes.c_int),
    "hkv_sync_check": ([_P, _P], ctypes.c_int),
    "hkv_rope_tables": ([_P, _P, _P], ctypes.c_int),
    "hkv_decode_attn_noalloc": ([ctypes.POINTER(PagedView), _I32, _I32, _I32P, _I32P, _I32P,
                                 _P, _P, _P, ctypes.c_char_p, ctypes.c_size_t], ctypes.c_int),
    "hkv_decode_attn_noalloc_sync_check": ([_P, ctypes.c_char_p, ctypes.c_size_t], ctypes.c_int),
    "hkv_split_export": ([_P, _I32, _I32, _P], ctypes.c_int),
    "hkv_split_connect": ([_P, _P], ctypes.c_int),
    "hkv_split_step": ([_P, _I32, _I32, _I32P, _P, _P, _P, _P], ctypes.c_int),
    "hkv_split_wait": ([_P, _I32, _P], ctypes.c_int),
    "hkv_split_output": ([_P, _I32, ctypes.POINTER(_P), _I64P], ctypes.c_int),
    "hkv_engine_config": ([_P, ctypes.POINTER(Config)], ctypes.c_int),
    "hkv_q4k_quantize": ([_P, _I64, _I64, _P, _P, ctypes.c_char_p, ctypes.c_size_t], ctypes.c_int),
    "hkv_q4k_gemv": ([ctypes.POINTER(Q4kGemvArgs), _P, ctypes.c_char_p, ctypes.c_size_t],
                     ctypes.c_int),
    "hkv_q4k_qkv": ([ctypes.POINTER(Q4kQkvArgs), _P, ctypes.c_char_p, ctypes.c_size_t],
                    ctypes.c_int),
    "hkv_q4k_sync_check": ([_P, ctypes.c_char_p, ctypes.c_size_t], ctypes.c_int),
    "hkv_backbone_create": ([_P, ctypes.POINTER(BackboneWeights), _I32, ctypes.POINTER(_P)],
                            ctypes.c_int),
    "hkv_backbone_destroy": ([_P], None),
    "hkv_backbone_last_error": ([_P], ctypes.c_char_p),
    "hkv_backbone_embed_text": ([_P, _I32, _I32P, _P], ctypes.c_int),
    "hkv_backbone_embed_codes": ([_P, _I32, _P, _P], ctypes.c_int),
    "hkv_backbone_decode": ([_P, _I32, _I32P, _I32, _P], ctypes.c_int),
    "hkv_backbone_buffers": ([_P, ctypes.POINTER(_P), ctypes.POINTER(_P), ctypes.POINTER(_P)],
                             ctypes.c_int),
    "hkv_backbone_sync_check": ([_P, _P], ctypes.c_int),
    "hkv_backbone_kernel_launches": ([_P, _I64P], ctypes.c_int),
    "hkv_profile_enable": ([_P, ctypes.c_int], ctypes.c_int),
    "hkv_profile_reset": ([_P], ctypes.c_int),
    "hkv_profile_read": ([_P, ctypes.c_int, _I64P, ctypes.POINTER(ctypes.c_double)], ctypes.c_int),
    "hkv_host_stats": ([_P, _I64P, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double),
                        ctypes.c_int], ctypes.c_int),
}

_lib: Optional[ctypes.CDLL] = None


def load_library(path: Optional[os.PathLike] = None) -> ctypes.CDLL:
    """Loads libhkv.so and declares every entry point; raises if absent."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise ImportError(
            f"{p} is missing: build it with `python higgs-audio.cpp_b200/hkv_build.py` "
            "(the engine has no fallback implementation)")
    lib = ctypes.CDLL(str(p))
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    if path is None:
        _lib = lib
    return lib


def _ptr(x) -> Optional[int]:
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return int(x.data_ptr())
    if isinstance(x, np.ndarray):
        return int(x.ctypes.data)
    raise TypeError(f"cannot take a device pointer from {type(x)!r}")


def _stream(s) -> Optional[int]:
    if s is None or s == 0:
        return None
    if isinstance(s, int):
        return s
    if hasattr(s, "cuda_stream"):
        return int(s.cuda_stream)
    raise TypeError(f"cannot take a CUDA stream handle from {type(s)!r}")


def _slots_arg(slots: Sequence[int]):
    arr = (ctypes.c_int32 * len(slots))(*[int(s) for s in slots])
    return len(slots), arr


class ScopedBackendKvCacheSlot:
    """RAII slot lease (ScopedBackendKvCacheSlot, src/higgs_pipeline.cpp:372-403)."""

    def __init__(self, engine: "Engine", slot: int):
        self.engine = engine
        self.slot = slot

    def release(self) -> None:
        if self.engine is not None and self.slot >= 0:
            self.engine.release(self.slot)
        self.engine = None
        self.slot = -1

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.release()
        return False


class Engine:
    """One paged KV engine (one page pool on one GPU, or host-only if device=-1)."""

    def __init__(self, n_layers: int = 36, n_head: int = 32, n_head_kv: int = 8,
                 head_dim: int = 128, page_tokens: int = 16, context_length: int = 32768,
                 rope_freq_base: float = 1e6, max_slots: int = 256, n_pages: int = 4096,
                 device: int = 0, shuffle_seed: int = 0, lib: Optional[ctypes.CDLL] = None):
        self.lib = lib or load_library()
        self.handle = None
        self.cfg = Config(n_layers, n_head, n_head_kv, head_dim, page_tokens, context_length,
                          rope_freq_base, max_slots, n_pages, device, shuffle_seed)
        h = ctypes.c_void_p()
        st = self.lib.hkv_engine_create(ctypes.byref(self.cfg), ctypes.byref(h))
        if st != HKV_OK:
            raise HkvError(st, f"hkv_engine_create failed: "
                               f"{self.lib.hkv_status_string(st).decode()}")
        self.handle = h

    # ---------------------------------------------------------------- misc
    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.hkv_engine_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
        return False

    def last_error(self) -> str:
        return self.lib.hkv_last_error(self.handle).decode()

    def _check(self, st: int) -> None:
        if st == HKV_OK:
            return
        msg = self.last_error()
        if st == HKV_ERR_RANGE:
            raise HkvRangeError(st, msg)
        raise HkvError(st, msg)

    # --------------------------------------------------------------- slots
    def acquire(self, capacity: int = 0, share: Optional[tuple] = None) -> int:
        out = ctypes.c_int32()
        key = PrefixKey(*share) if share is not None else None
        self._check(self.lib.hkv_slot_acquire(self.handle, capacity,
                                              ctypes.byref(key) if key else None,
                                              ctypes.byref(out)))
        return out.value

    def acquire_backend_kv_cache_slot(self, capacity: int,
                                      share: Optional[tuple] = None) -> ScopedBackendKvCacheSlot:
        return ScopedBackendKvCacheSlot(self, self.acquire(capacity, share))

    def release(self, slot: int) -> None:
        self._check(self.lib.hkv_slot_release(self.handle, slot))

    def fork(self, src: int, n_tokens: int) -> int:
        out = ctypes.c_int32()
        self._check(self.lib.hkv_slot_fork(self.handle, src, n_tokens, ctypes.byref(out)))
        return out.value

    def length(self, slot: int) -> int:
        out = ctypes.c_int64()
        self._check(self.lib.hkv_slot_len(self.handle, slot, ctypes.byref(out)))
        return out.value

    def set_length(self, slot: int, used: int) -> None:
        self._check(self.lib.hkv_slot_set_len(self.handle, slot, used))

    def advance(self, slots: Sequence[int], n_tokens: int = 1) -> None:
        n, arr = _slots_arg(slots)
        self._check(self.lib.hkv_slot_advance(self.handle, n, arr, n_tokens))

    def publish(self, key_hash: int, n_tokens: int, slot: int) -> None:
        key = PrefixKey(key_hash, n_tokens)
        self._check(self.lib.hkv_prefix_publish(self.handle, ctypes.byref(key), slot))

    def drop(self, key_hash: int, n_tokens: int) -> None:
        key = PrefixKey(key_hash, n_tokens)
        self._check(self.lib.hkv_prefix_drop(self.handle, ctypes.byref(key)))

    def pages(self, slot: int) -> list:
        n = ctypes.c_int64()
        self._check(self.lib.hkv_slot_pages(self.handle, slot, None, 0, ctypes.byref(n)))
        buf = (ctypes.c_int32 * max(1, n.value))()
        self._check(self.lib.hkv_slot_pages(self.handle, slot, buf, n.value, ctypes.byref(n)))
        return list(buf[: n.value])

    def stats(self) -> dict:
        s = PoolStats()
        self._check(self.lib.hkv_pool_stats_get(self.handle, ctypes.byref(s)))
        return {f: getattr(s, f) for f, _ in PoolStats._fields_}

    # ------------------------------------------------------------- compute
    def append(self, layer: int, slots: Sequence[int], k, v, stream=None) -> None:
        n, arr = _slots_arg(slots)
        self._check(self.lib.hkv_append(self.handle, layer, n, arr, _ptr(k), _ptr(v),
                                        _stream(stream)))

    def rope_append(self, layer: int, slots: Sequence[int], k, v, stream=None) -> None:
        n, arr = _slots_arg(slots)
        self._check(self.lib.hkv_rope_append(self.handle, layer, n, arr, _ptr(k), _ptr(v),
                                             _stream(stream)))

    def rope_append_range(self, layer: int, slot: int, n_tokens: int, k, v, stream=None) -> None:
        self._check(self.lib.hkv_rope_append_range(self.handle, layer, slot, n_tokens, _ptr(k),
                                                   _ptr(v), _stream(stream)))

    def decode_attn(self, layer: int, slots: Sequence[int], q, out, stream=None) -> None:
        n, arr = _slots_arg(slots)
        self._check(self.lib.hkv_decode_attn(self.handle, layer, n, arr, _ptr(q), _ptr(out),
                                             _stream(stream)))

    def decode_step(self, layer: int, slots: Sequence[int], q, k, v, out, stream=None) -> None:
        n, arr = _slots_arg(slots)
        self._check(self.lib.hkv_decode_step(self.handle, layer, n, arr, _ptr(q), _ptr(k),
                                             _ptr(v), _ptr(out), _stream(stream)))

    def gather(self, slot: int, layer: int, pos0: int, n: int, k_out, v_out, stream=None) -> None:
        self._check(self.lib.hkv_gather(self.handle, slot, layer, pos0, n, _ptr(k_out),
                                        _ptr(v_out), _stream(stream)))

    def sync_check(self, stream=None) -> None:
        self._check(self.lib.hkv_sync_check(self.handle, _stream(stream)))

    def slots_array(self, slots: Sequence[int]):
        """(n, ctypes int32 array) of a slot list, for decode_step_ptrs."""
        return _slots_arg(slots)

    def decode_step_ptrs(self, layer: int, n: int, slots_arr, q: int, k: int, v: int, out: int,
                         stream: int) -> None:
        """hkv_decode_step with every argument prepared (device pointers and the
        stream as ints, the slots as a ctypes array): the least a caller does
        per call."""
        st = self.lib.hkv_decode_step(self.handle, layer, n, slots_arr, q, k, v, out, stream)
        if st != HKV_OK:
            self._check(st)

    def host_stats(self, reset: bool = False):
        """(calls, host microseconds, of which launch calls and buffer waits that
        can block on the GPU) spent in hkv_decode_step / hkv_decode_attn."""
        c = ctypes.c_int64()
        us = ctypes.c_double()
        lus = ctypes.c_double()
        self._check(self.lib.hkv_host_stats(self.handle, ctypes.byref(c), ctypes.byref(us),
                                            ctypes.byref(lus), 1 if reset else 0))
        return c.value, us.value, lus.value

    def rope_tables(self):
        half = self.cfg.head_dim // 2
        cos = np.empty((self.cfg.context_length, half), np.float32)
        sin = np.empty_like(cos)
        self._check(self.lib.hkv_rope_tables(self.handle, cos.ctypes.data, sin.ctypes.data))
        return cos, sin

    # ------------------------------------------------------- KV-head split
    def split_export(self, world: int, rank: int) -> bytes:
        buf = ctypes.create_string_buffer(64)
        self._check(self.lib.hkv_split_export(self.handle, world, rank, buf))
        return buf.raw

    def split_connect(self, handles: Sequence[bytes]) -> None:
        blob = b"".join(handles)
        buf = ctypes.create_string_buffer(blob, len(blob))
        self._check(self.lib.hkv_split_connect(self.handle, buf))

    def split_disconnect(self) -> None:
        self._check(self.lib.hkv_split_connect(self.handle, None))

    def split_step(self, layer: int, slots: Sequence[int], q, k, v, stream=None) -> None:
        n, arr = _slots_arg(slots)
        self._check(self.lib.hkv_split_step(self.handle, layer, n, arr, _ptr(q), _ptr(k), _ptr(v),
                                            _stream(stream)))

    def split_wait(self, layer: int, stream=None) -> None:
        self._check(self.lib.hkv_split_wait(self.handle, layer, _stream(stream)))

    def split_output(self, layer: int):
        """(device pointer, floats per row) of this rank's full output of one layer."""
        p = ctypes.c_void_p()
        w = ctypes.c_int64()
        self._check(self.lib.hkv_split_output(self.handle, layer, ctypes.byref(p), ctypes.byref(w)))
        return p.value, w.value

    # ----------------------------------------------------------- profiling
    def profile_enable(self, on: bool = True) -> None:
        self._check(self.lib.hkv_profile_enable(self.handle, 1 if on else 0))

    def profile_reset(self) -> None:
        self._check(self.lib.hkv_profile_reset(self.handle))

    def profile_read(self, kernel_id: int):
        n = ctypes.c_int64()
        ms = ctypes.c_double()
        self._check(self.lib.hkv_profile_read(self.handle, kernel_id, ctypes.byref(n),
                                              ctypes.byref(ms)))
        return n.value, ms.value


def decode_attn_noalloc(view: PagedView, layer: int, pos: Sequence[int],
                        page_lists: Sequence[Sequence[int]], q, out, stream=None,
                        lib: Optional[ctypes.CDLL] = None) -> None:
    """hkv_decode_attn_noalloc: attention over caller-owned pages, no device
    allocation.  page_lists[e] are slot e's physical pages."""
    lib = lib or load_library()
    n = len(pos)
    offs = [0]
    for pl in page_lists:
        offs.append(offs[-1] + len(pl))
    flat = [int(p) for pl in page_lists for p in pl]
    msg = ctypes.create_string_buffer(512)
    st = lib.hkv_decode_attn_noalloc(
        ctypes.byref(view), layer, n, (ctypes.c_int32 * n)(*[int(p) for p in pos]),
        (ctypes.c_int32 * (n + 1))(*offs), (ctypes.c_int32 * max(1, len(flat)))(*flat),
        _ptr(q), _ptr(out), _stream(stream), msg, len(msg))
    if st != HKV_OK:
        cls = HkvRangeError if st == HKV_ERR_RANGE else HkvError
        raise cls(st, msg.value.decode())


def decode_attn_noalloc_sync_check(stream=None, lib: Optional[ctypes.CDLL] = None) -> None:
    """hkv_decode_attn_noalloc_sync_check: synchronise `stream` and raise if a
    no-allocation call recorded a device-side error since the last check."""
    lib = lib or load_library()
    msg = ctypes.create_string_buffer(512)
    _raise_msg(lib.hkv_decode_attn_noalloc_sync_check(_stream(stream), msg, len(msg)), msg)


class DeviceArray:
    """A raw device pointer exposed through __cuda_array_interface__ (wrap it
    with torch.as_tensor(..., device=...) to read an engine buffer)."""

    def __init__(self, ptr: int, shape, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3, "strides": None}


# --------------------------------------------------------- Q4_K backbone
def _raise_msg(st: int, msg) -> None:
    if st != HKV_OK:
        cls = HkvRangeError if st == HKV_ERR_RANGE else HkvError
        raise cls(st, msg.value.decode())


def q4k_quantize(w, rows: int, cols: int, blocks, stream=None, lib=None) -> None:
    """hkv_q4k_quantize: F32 [rows][cols] device -> Q4_K blocks (rows*cols/256*144 bytes)."""
    lib = lib or load_library()
    msg = ctypes.create_string_buffer(512)
    _raise_msg(lib.hkv_q4k_quantize(_ptr(w), rows, cols, _ptr(blocks), _stream(stream), msg,
                                    len(msg)), msg)


def q4k_gemv(w, rows: int, cols: int, x, y, n: int = 1, norm=None, eps: float = 1e-6,
             residual=None, w_up=None, stream=None, lib=None, tensor_cores: bool = False) -> None:
    """hkv_q4k_gemv: y = [residual +] W x' or silu(W x') * (W_up x');
    tensor_cores: the tensor-core kernel even for n == 1."""
    lib = lib or load_library()
    a = Q4kGemvArgs(_ptr(w), _ptr(w_up), rows, cols, n, _ptr(x), _ptr(norm), eps, _ptr(residual),
                    _ptr(y), 1 if tensor_cores else 0)
    msg = ctypes.create_string_buffer(512)
    _raise_msg(lib.hkv_q4k_gemv(ctypes.byref(a), _stream(stream), msg, len(msg)), msg)


def q4k_qkv(wq, wk, wv, cols: int, x, q_norm, k_norm, q_out, k_out, v_out, n: int = 1,
            norm=None, eps: float = 1e-6, n_head: int = 32, n_head_kv: int = 8, stream=None,
            lib=None, tensor_cores: bool = False) -> None:
    """hkv_q4k_qkv: q/k/v projections with the per-head norms of q and k."""
    lib = lib or load_library()
    a = Q4kQkvArgs(_ptr(wq), _ptr(wk), _ptr(wv), n_head, n_head_kv, cols, n, _ptr(x), _ptr(norm),
                   eps, _ptr(q_norm), _ptr(k_norm), _ptr(q_out), _ptr(k_out), _ptr(v_out),
                   1 if tensor_cores else 0)
    msg = ctypes.create_string_buffer(512)
    _raise_msg(lib.hkv_q4k_qkv(ctypes.byref(a), _stream(stream), msg, len(msg)), msg)


def q4k_sync_check(stream=None, lib=None) -> None:
    """hkv_q4k_sync_check: synchronise and report a timed-out projection launch."""
    lib = lib or load_library()
    msg = ctypes.create_string_buffer(512)
    _raise_msg(lib.hkv_q4k_sync_check(_stream(stream), msg, len(msg)), msg)


class Backbone:
    """hkv_backbone: the Q4_K decode step around an engine.  `weights` maps
    names to device tensors (kept referenced here): per layer l
    "blk.{l}.attn_q" ... "blk.{l}.attn_k_norm", plus "token_embd",
    "a.token_embd", "output_norm", "a.output"."""

    LAYER_KEYS = ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down",
                  "attn_norm", "ffn_norm", "attn_q_norm", "attn_k_norm")

    def __init__(self, engine: "Engine", weights: dict, hidden: int = 2560, ffn: int = 9728,
                 text_vocab: int = 151936, n_codebooks: int = 8, codebook_size: int = 1026,
                 rms_eps: float = 1e-6, max_batch: int = 1):
        self.engine = engine
        self.lib = engine.lib
        self.weights = weights
        n_layers = engine.cfg.n_layers
        self._layers = (BackboneLayer * n_layers)()
        for l in range(n_layers):
            for key in self.LAYER_KEYS:
                setattr(self._layers[l], key, _ptr(weights[f"blk.{l}.{key}"]))
        self._w = BackboneWeights(hidden, ffn, text_vocab, n_codebooks, codebook_size, rms_eps,
                                  self._layers, _ptr(weights["token_embd"]),
                                  _ptr(weights["a.token_embd"]), _ptr(weights["output_norm"]),
                                  _ptr(weights["a.output"]))
        h = ctypes.c_void_p()
        st = self.lib.hkv_backbone_create(engine.handle, ctypes.byref(self._w), max_batch,
                                          ctypes.byref(h))
        if st != HKV_OK:
            raise HkvError(st, f"hkv_backbone_create failed: status {st}")
        self.handle = h
        self.n_codebooks, self.codebook_size, self.hidden = n_codebooks, codebook_size, hidden
        hp, lp, cp = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        self.lib.hkv_backbone_buffers(self.handle, ctypes.byref(hp), ctypes.byref(lp),
                                      ctypes.byref(cp))
        self.hidden_ptr, self.logits_ptr, self.codes_ptr = hp.value, lp.value, cp.value

    def _check(self, st: int) -> None:
        if st != HKV_OK:
            msg = self.lib.hkv_backbone_last_error(self.handle).decode()
            cls = HkvRangeError if st == HKV_ERR_RANGE else HkvError
            raise cls(st, msg)

    def embed_text(self, ids: Sequence[int], stream=None) -> None:
        n, arr = _slots_arg(ids)
        self._check(self.lib.hkv_backbone_embed_text(self.handle, n, arr, _stream(stream)))

    def embed_codes(self, n: int, codes=None, stream=None) -> None:
        self._check(self.lib.hkv_backbone_embed_codes(self.handle, n, _ptr(codes), _stream(stream)))

    def decode(self, slots: Sequence[int], want_logits: bool = True, stream=None) -> None:
        n, arr = _slots_arg(slots)
        self._check(self.lib.hkv_backbone_decode(self.handle, n, arr, 1 if want_logits else 0,
                                                 _stream(stream)))

    def sync_check(self, stream=None) -> None:
        self._check(self.lib.hkv_backbone_sync_check(self.handle, _stream(stream)))

    @property
    def kernel_launches(self) -> int:
        """Kernels this backbone has launched (embedding, projections, argmax)."""
        v = ctypes.c_int64(0)
        self._check(self.lib.hkv_backbone_kernel_launches(self.handle, ctypes.byref(v)))
        return v.value

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.hkv_backbone_destroy(self.handle)
            self.handle = None


def header_functions(header: Path) -> list:
    """Names of the functions a C header declares."""
    text = Path(header).read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(hkv_[a-z0-9_]+)\s*\(", text)))
