"""ctypes view of the CPU oracle (oracle/hkv_oracle.c, oracle/hkv_oracle_graph.c).

TEST AND MEASUREMENT INFRASTRUCTURE.  Imported only by tests/, by
__graft_entry__.smoke() as the reference result, and by bench.py's CPU-baseline leg and
`--impl reference` arm.  The engine never imports it.

Pinning (see the C file header): append and layout are pinned by the
reference's known-answer self-checks; the RoPE table formula is compared with
the reference's own table code compiled from its source (oracle/_ref, when the
reference checkout is present); the attention numerics are parity-unpinned.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"

EXACT = 0
GGML_F16 = 1

_lib = None


def build(force: bool = False) -> Path:
    """Compiles the oracle with the committed Makefile (gcc, OpenMP)."""
    srcs = [HERE / "hkv_oracle.c", HERE / "hkv_oracle_q4k.c", HERE / "hkv_oracle_graph.c",
            HERE / "Makefile"]
    if force or not LIB_PATH.exists() or any(
            s.stat().st_mtime > LIB_PATH.stat().st_mtime for s in srcs):
        subprocess.run(["make", "-s", "-C", str(HERE), "-B" if force else "all"], check=True)
    return LIB_PATH


def reference_checkout():
    """Location of a checkout of the reference (bluryar/higgs-audio.cpp), or
    None: the HKV_REFERENCE environment variable, else a directory named
    `reference` beside this repository.  Only the RoPE-table pin
    (oracle/ref_rope_table.sh) reads it."""
    import os
    env = os.environ.get("HKV_REFERENCE")
    cands = [Path(env)] if env else [HERE.parents[1] / "reference"]
    for c in cands:
        if (c / "src" / "higgs_pipeline.cpp").is_file():
            return c
    return None


def build_reference_table_code() -> bool:
    """Compiles the reference's own RoPE-table code into oracle/_ref/ when a
    checkout is available; returns False (with a message) when it is not."""
    ref = reference_checkout()
    if ref is None:
        print("oracle/_ref not built: no reference checkout (set HKV_REFERENCE); the RoPE "
              "table stays pinned by tests/golden/rope_table_ref.npz")
        return False
    subprocess.run([str(HERE / "ref_rope_table.sh"), str(ref)], check=True,
                   stdout=subprocess.DEVNULL)
    return True


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        P = ctypes.c_void_p
        I64 = ctypes.c_int64
        L.hkvo_bf16_round.argtypes = [ctypes.c_float]
        L.hkvo_bf16_round.restype = ctypes.c_float
        L.hkvo_rope_table.argtypes = [I64, I64, ctypes.c_float, P, P]
        L.hkvo_f32_to_f16.argtypes = [ctypes.c_float]
        L.hkvo_f32_to_f16.restype = ctypes.c_uint16
        L.hkvo_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.hkvo_f16_to_f32.restype = ctypes.c_float
        L.hkvo_f32_to_f16_array.argtypes = [P, P, I64]
        L.hkvo_f16_to_f32_array.argtypes = [P, P, I64]
        L.hkvo_rope_neox.argtypes = [P, I64, I64, P, P, P]
        L.hkvo_append_rows.argtypes = [I64, I64, I64, P, P, P, P, P, ctypes.c_int, P, P]
        L.hkvo_decode_attn.argtypes = [ctypes.c_int, I64, I64, I64, I64, P, P, P, P, P,
                                       ctypes.c_float, P]
        L.hkvo_graph_decode_layer.argtypes = [I64, I64, I64, I64, P, P, P, P, P, P, P, P, P,
                                              ctypes.c_float, P, P]
        L.hkvo_graph_work_floats.argtypes = [I64, I64, I64, I64]
        L.hkvo_graph_work_floats.restype = I64
        L.hkvo_q4k_dequant.argtypes = [P, I64, P]
        L.hkvo_q8k_quantize.argtypes = [P, I64, P]
        L.hkvo_q4k_dot_q8k.argtypes = [P, P, I64]
        L.hkvo_q4k_dot_q8k.restype = ctypes.c_float
        L.hkvo_q4k_gemv.argtypes = [P, I64, I64, P, I64, P, P]
        L.hkvo_rms_norm_mul.argtypes = [P, I64, I64, ctypes.c_float, P, P]
        L.hkvo_silu_mul.argtypes = [P, P, I64, P]
        L.hkvo_max_threads.restype = ctypes.c_int
        L.hkvo_set_threads.argtypes = [ctypes.c_int]
        _lib = L
    return _lib


def _p(a: np.ndarray) -> int:
    assert a.flags.c_contiguous
    return a.ctypes.data


def scale(head_dim: int = 128) -> float:
    """1/sqrt(head_dim) in F32, as the reference computes it (:5767)."""
    return float(np.float32(1.0) / np.sqrt(np.float32(head_dim)))


def rope_table(context_length: int = 32768, key_length: int = 128, base: float = 1e6):
    half = key_length // 2
    cos = np.empty((context_length, half), np.float32)
    sin = np.empty_like(cos)
    lib().hkvo_rope_table(context_length, key_length, base, _p(cos), _p(sin))
    return cos, sin


def bf16_round(x: float) -> float:
    return lib().hkvo_bf16_round(x)


def f32_to_f16(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    out = np.empty(a.shape, np.uint16)
    lib().hkvo_f32_to_f16_array(_p(a), _p(out), a.size)
    return out


def f16_to_f32(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, np.uint16)
    out = np.empty(a.shape, np.float32)
    lib().hkvo_f16_to_f32_array(_p(a), _p(out), a.size)
    return out


def rope_neox(x: np.ndarray, cos_row: np.ndarray, sin_row: np.ndarray) -> np.ndarray:
    """x: [n_head][head_dim] F32 at one position."""
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().hkvo_rope_neox(_p(x), x.shape[0], x.shape[1], _p(np.ascontiguousarray(cos_row)),
                         _p(np.ascontiguousarray(sin_row)), _p(y))
    return y


def append_rows(k: np.ndarray, v: np.ndarray, pos: np.ndarray, cos: np.ndarray,
                sin: np.ndarray, rope: bool = True):
    """F16 bits the cache must hold after appending rows k (pre-RoPE), v.

    k, v: [n][n_head_kv][head_dim] F32; pos: [n] positions."""
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    pos = np.ascontiguousarray(pos, np.int32)
    ko = np.empty(k.shape, np.uint16)
    vo = np.empty(v.shape, np.uint16)
    lib().hkvo_append_rows(k.shape[0], k.shape[1], k.shape[2], _p(k), _p(v), _p(pos), _p(cos),
                           _p(sin), 1 if rope else 0, _p(ko), _p(vo))
    return ko, vo


def decode_attn(q_roped: np.ndarray, k_caches, v_caches, mode: int = EXACT) -> np.ndarray:
    """Attention of one token per slot over logical F16 caches.

    q_roped: [n][n_head][head_dim] F32; k_caches/v_caches: list of
    [L_e][n_head_kv][head_dim] uint16 arrays.  Returns [n][n_head*head_dim]."""
    q = np.ascontiguousarray(q_roped, np.float32)
    n, H, D = q.shape
    G = k_caches[0].shape[1]
    lens = np.array([c.shape[0] for c in k_caches], np.int32)
    row_off = np.zeros(n, np.int64)
    row_off[1:] = np.cumsum(lens[:-1])
    k_all = np.ascontiguousarray(np.concatenate(k_caches, 0), np.uint16)
    v_all = np.ascontiguousarray(np.concatenate(v_caches, 0), np.uint16)
    out = np.empty((n, H * D), np.float32)
    lib().hkvo_decode_attn(mode, n, H, G, D, _p(q), _p(k_all), _p(v_all), _p(row_off), _p(lens),
                           scale(D), _p(out))
    return out


def decode_attn_rows(q_roped: np.ndarray, k_all: np.ndarray, v_all: np.ndarray,
                     row_off: np.ndarray, lens: np.ndarray, mode: int = EXACT) -> np.ndarray:
    """decode_attn over caches kept in one array: slot e's rows are
    k_all[row_off[e] : row_off[e] + lens[e]] (uint16 [rows][n_head_kv][head_dim]),
    so large caches are not copied per call."""
    q = np.ascontiguousarray(q_roped, np.float32)
    n, H, D = q.shape
    G = k_all.shape[1]
    assert k_all.flags.c_contiguous and v_all.flags.c_contiguous
    assert k_all.dtype == np.uint16 and v_all.dtype == np.uint16
    row_off = np.ascontiguousarray(row_off, np.int64)
    lens = np.ascontiguousarray(lens, np.int32)
    assert row_off.shape == (n,) and lens.shape == (n,)
    assert np.all(row_off >= 0) and np.all(row_off + lens <= k_all.shape[0])
    out = np.empty((n, H * D), np.float32)
    lib().hkvo_decode_attn(mode, n, H, G, D, _p(q), _p(k_all), _p(v_all), _p(row_off), _p(lens),
                           scale(D), _p(out))
    return out


class GraphBaseline:
    """The reference's F32 decode graph for one layer over contiguous per-slot
    caches (hkv_oracle_graph.c): the timed CPU baseline."""

    def __init__(self, n_slots: int, capacity: int, n_head: int = 32, n_head_kv: int = 8,
                 head_dim: int = 128, cos=None, sin=None, fill_seed=None):
        self.n, self.cap, self.H, self.G, self.D = n_slots, capacity, n_head, n_head_kv, head_dim
        if fill_seed is None:
            self.k_cache = np.zeros((n_slots * capacity, n_head_kv, head_dim), np.float32)
            self.v_cache = np.zeros_like(self.k_cache)
        else:
            # N(0,1) rows: a seeded block tiled over the whole cache (fast to
            # fill; the graph's cost does not depend on the values)
            block = np.random.default_rng(fill_seed).standard_normal(
                (4096, n_head_kv, head_dim), dtype=np.float32)
            rows = n_slots * capacity
            self.k_cache = np.empty((rows, n_head_kv, head_dim), np.float32)
            self.v_cache = np.empty_like(self.k_cache)
            for a in range(0, rows, 4096):
                b = min(rows, a + 4096)
                self.k_cache[a:b] = block[:b - a]
                self.v_cache[a:b] = block[::-1][:b - a]
        self.row_off = (np.arange(n_slots, dtype=np.int64) * capacity)
        work = lib().hkvo_graph_work_floats(capacity, n_head, n_head_kv, head_dim)
        self.work = np.zeros(int(work), np.float32)
        if cos is None:
            cos, sin = rope_table(key_length=head_dim)
        self.cos, self.sin = np.ascontiguousarray(cos), np.ascontiguousarray(sin)
        self.out = np.zeros((n_slots, n_head * head_dim), np.float32)

    def decode_layer(self, q_pre, k_pre, v_new, past) -> np.ndarray:
        """One layer for the first len(past) slots."""
        past = np.ascontiguousarray(past, np.int32)
        n = past.shape[0]
        assert 0 < n <= self.n and past.max() < self.cap
        q_pre = np.ascontiguousarray(q_pre, np.float32)
        k_pre = np.ascontiguousarray(k_pre, np.float32)
        v_new = np.ascontiguousarray(v_new, np.float32)
        assert q_pre.shape[0] == n and k_pre.shape[0] == n and v_new.shape[0] == n
        lib().hkvo_graph_decode_layer(n, self.H, self.G, self.D, _p(q_pre), _p(k_pre),
                                      _p(v_new), _p(self.k_cache), _p(self.v_cache),
                                      _p(self.row_off), _p(past), _p(self.cos), _p(self.sin),
                                      scale(self.D), _p(self.work), _p(self.out))
        return self.out


# ------------------------------------------------------------ Q4_K backbone
Q4K_BYTES = 144  # bytes of one 256-weight Q4_K block
Q8K_BYTES = 292  # bytes of one 256-activation Q8_K block


def q4k_dequant(blocks: np.ndarray, cols: int) -> np.ndarray:
    """Q4_K bytes [rows][cols/256*144] -> F32 [rows][cols]."""
    blocks = np.ascontiguousarray(blocks, np.uint8)
    n_blocks = blocks.size // Q4K_BYTES
    out = np.empty(n_blocks * 256, np.float32)
    lib().hkvo_q4k_dequant(_p(blocks), n_blocks, _p(out))
    return out.reshape(-1, cols)


def q8k_quantize(x: np.ndarray) -> np.ndarray:
    """F32 [..., k] -> Q8_K bytes [..., k/256*292]."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.size // 256 * Q8K_BYTES, np.uint8)
    lib().hkvo_q8k_quantize(_p(x), x.size, _p(out))
    return out.reshape(x.shape[:-1] + (x.shape[-1] // 256 * Q8K_BYTES,))


def q8k_dequant(blocks: np.ndarray) -> np.ndarray:
    """Q8_K bytes -> F32 (d * q), for checks."""
    b = np.ascontiguousarray(blocks, np.uint8).reshape(-1, Q8K_BYTES)
    d = b[:, :4].copy().view(np.float32)
    q = b[:, 4:260].view(np.int8).astype(np.float32)
    return (q * d).reshape(-1)


def q4k_dot_q8k(w_row: np.ndarray, a: np.ndarray) -> float:
    w_row = np.ascontiguousarray(w_row, np.uint8)
    a = np.ascontiguousarray(a, np.uint8)
    return float(lib().hkvo_q4k_dot_q8k(_p(w_row), _p(a), w_row.size // Q4K_BYTES))


def q4k_gemv(w: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    """mul_mat_f32(W, x) with Q4_K W: x [n][cols] F32 -> [n][rows]."""
    w = np.ascontiguousarray(w, np.uint8)
    x = np.ascontiguousarray(x, np.float32).reshape(-1, cols)
    n = x.shape[0]
    y = np.empty((n, rows), np.float32)
    scratch = np.empty(n * (cols // 256) * Q8K_BYTES, np.uint8)
    lib().hkvo_q4k_gemv(_p(w), rows, cols, _p(x), n, _p(y), _p(scratch))
    return y


def rms_norm_mul(x: np.ndarray, eps: float, weight=None) -> np.ndarray:
    """ggml_rms_norm over the last axis, then ggml_mul by `weight`."""
    x = np.ascontiguousarray(x, np.float32)
    n = x.shape[-1]
    y = np.empty_like(x)
    w = None if weight is None else np.ascontiguousarray(weight, np.float32)
    lib().hkvo_rms_norm_mul(_p(x), x.size // n, n, eps, None if w is None else _p(w), _p(y))
    return y


def silu_mul(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    gate = np.ascontiguousarray(gate, np.float32)
    up = np.ascontiguousarray(up, np.float32)
    y = np.empty_like(gate)
    lib().hkvo_silu_mul(_p(gate), _p(up), gate.size, _p(y))
    return y


def max_threads() -> int:
    return lib().hkvo_max_threads()


def set_threads(n: int) -> None:
    lib().hkvo_set_threads(n)


class BackboneOracle:
    """The reference's per-frame decode graph on the CPU
    (run_kv_decode_graph_all_layers_with_backend_cache_ex,
    src/higgs_pipeline.cpp:5629-5863) with Q4_K weights and the engine's F16
    KV rows: rms_norm * attn_norm -> Q4_K q/k/v (Q8_K activations) -> per-head
    rms_norm * q_norm / k_norm -> RoPE -> append -> attention -> h + Wo attn ->
    rms_norm * ffn_norm -> silu(Wg m) * (Wu m) -> h + Wd g; then
    a.output(rms_norm(h) * output_norm) and the first maximum per codebook.

    `weights` maps the GGUF names to numpy arrays: Q4_K matrices as uint8
    [rows][cols/256*144], norms as float32."""

    def __init__(self, weights: dict, n_layers: int, hidden: int = 2560, ffn: int = 9728,
                 n_head: int = 32, n_head_kv: int = 8, head_dim: int = 128, n_codebooks: int = 8,
                 codebook_size: int = 1026, eps: float = 1e-6, cos=None, sin=None):
        self.w = weights
        self.L, self.hidden, self.ffn = n_layers, hidden, ffn
        self.H, self.G, self.D = n_head, n_head_kv, head_dim
        self.nc, self.cs, self.eps = n_codebooks, codebook_size, eps
        if cos is None:
            cos, sin = rope_table(key_length=head_dim)
        self.cos, self.sin = cos, sin
        self.caches = {}  # (slot, layer) -> (k rows, v rows) as uint16 [R][G][D]

    def embed_text(self, ids) -> np.ndarray:
        t = self.w["token_embd"]
        return np.stack([q4k_dequant(t[i], self.hidden)[0] for i in ids]).astype(np.float32)

    def embed_codes(self, codes) -> np.ndarray:
        t = self.w["a.token_embd"]
        out = []
        for row in np.asarray(codes).reshape(-1, self.nc):
            acc = None
            for c, code in enumerate(row):
                r = q4k_dequant(t[c * self.cs + int(code)], self.hidden)[0]
                acc = r if acc is None else (acc + r).astype(np.float32)
            out.append(acc)
        return np.stack(out).astype(np.float32)

    def _gemv(self, name: str, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
        return q4k_gemv(self.w[name], rows, cols, x)

    def decode(self, h: np.ndarray, slots, pos, want_logits: bool = True):
        """One token per slot at positions `pos`; returns (h, logits, codes)."""
        n = h.shape[0]
        H, G, D, eps = self.H, self.G, self.D, self.eps
        h = np.ascontiguousarray(h, np.float32)
        for l in range(self.L):
            p = f"blk.{l}."
            xn = rms_norm_mul(h, eps, self.w[p + "attn_norm"])
            q = self._gemv(p + "attn_q", H * D, self.hidden, xn).reshape(n, H, D)
            k = self._gemv(p + "attn_k", G * D, self.hidden, xn).reshape(n, G, D)
            v = self._gemv(p + "attn_v", G * D, self.hidden, xn).reshape(n, G, D)
            q = rms_norm_mul(q, eps, self.w[p + "attn_q_norm"])
            k = rms_norm_mul(k, eps, self.w[p + "attn_k_norm"])
            k16, v16 = append_rows(k, v, np.asarray(pos), self.cos, self.sin)
            ks, vs, qr = [], [], []
            for e, s in enumerate(slots):
                kc, vc = self.caches.get((s, l), (np.zeros((0, G, D), np.uint16),) * 2)
                kc = np.concatenate([kc[:pos[e]], k16[e:e + 1]])
                vc = np.concatenate([vc[:pos[e]], v16[e:e + 1]])
                self.caches[(s, l)] = (kc, vc)
                ks.append(kc)
                vs.append(vc)
                qr.append(rope_neox(q[e], self.cos[pos[e]], self.sin[pos[e]]))
            attn = decode_attn(np.stack(qr), ks, vs)
            h = (h + self._gemv(p + "attn_output", self.hidden, H * D, attn)).astype(np.float32)
            m = rms_norm_mul(h, eps, self.w[p + "ffn_norm"])
            g = silu_mul(self._gemv(p + "ffn_gate", self.ffn, self.hidden, m),
                         self._gemv(p + "ffn_up", self.ffn, self.hidden, m))
            h = (h + self._gemv(p + "ffn_down", self.hidden, self.ffn, g)).astype(np.float32)
        if not want_logits:
            return h, None, None
        logits = self._gemv("a.output", self.nc * self.cs, self.hidden,
                            rms_norm_mul(h, eps, self.w["output_norm"]))
        codes = logits.reshape(n, self.nc, self.cs).argmax(-1).astype(np.int32)
        return h, logits, codes
