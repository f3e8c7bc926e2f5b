"""Generates the committed golden fixtures in tests/golden/.

Run here, where the reference checkout is present:
    python tests/golden/make_golden.py

Fixtures:
  rope_table_ref.npz   rows of the BF16 RoPE table produced by the
                       reference's OWN table code (make_bf16_rope_table,
                       src/higgs_pipeline.cpp:475-487), compiled from its
                       source by oracle/ref_rope_table.sh, plus the SHA-256 of
                       the full [32768][64] cos and sin tables.
  append_selfcheck.npz the known-answer append of
                       self_check_backend_kv_cache_write (:6960-6986):
                       K[i] = i%17 + 0.25, V[i] = -(i%19) - 0.5 for one
                       [8][128] row written at layer 0, position 1 and read
                       back unchanged; the expected F16 bits come from numpy's
                       float16 (all values are exact in F16).
  layout_selfcheck.npz the front/back known answer of self_check_kv_cache
                       (:5206-5227): in a cache of capacity 4 the element
                       (layer 0, pos 0, head 0, dim 0) is flat index 0 and
                       (layer L-1, pos 3, head G-1, dim D-1) is the last one,
                       with per-layer logical rows [pos][head][dim].
  decode_seed.npz      deterministic inputs built from the reference's
                       self-check patterns (past K (i%31-15)/31 and V
                       (i%29-14)/29, :5338-5341; new K/V (i%23-11)/23,
                       :6996-6998; q (i%127-63)/63, :6690-6692) and the
                       oracle's outputs for them (a regression fixture: the
                       attention numerics themselves are parity-unpinned).
"""
from __future__ import annotations

import ctypes
import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO / "oracle"))
import cpu_oracle  # noqa: E402

CTX, KEY, BASE = 32768, 128, 1e6
ROWS = np.array([0, 1, 2, 3, 15, 16, 17, 100, 511, 512, 513, 1000, 2047, 4095, 4096, 8191,
                 16383, 16384, 32767], np.int64)


def reference_rope_table():
    so = REPO / "oracle" / "_ref" / "libref_rope.so"
    if not cpu_oracle.build_reference_table_code():
        raise SystemExit("rope_table_ref.npz needs a reference checkout (HKV_REFERENCE)")
    lib = ctypes.CDLL(str(so))
    lib.ref_rope_table.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_float,
                                   ctypes.c_void_p, ctypes.c_void_p]
    cos = np.empty((CTX, KEY // 2), np.float32)
    sin = np.empty_like(cos)
    lib.ref_rope_table(CTX, KEY, BASE, cos.ctypes.data, sin.ctypes.data)
    return cos, sin


def main():
    cpu_oracle.build()
    cos, sin = reference_rope_table()
    np.savez_compressed(
        HERE / "rope_table_ref.npz", rows=ROWS, cos_rows=cos[ROWS], sin_rows=sin[ROWS],
        cos_sha256=np.frombuffer(hashlib.sha256(cos.tobytes()).digest(), np.uint8),
        sin_sha256=np.frombuffer(hashlib.sha256(sin.tobytes()).digest(), np.uint8))

    i = np.arange(8 * 128)
    k = ((i % 17).astype(np.float32) + np.float32(0.25)).reshape(8, 128)
    v = (-(i % 19).astype(np.float32) - np.float32(0.5)).reshape(8, 128)
    np.savez_compressed(HERE / "append_selfcheck.npz", k=k, v=v, layer=0, pos=1,
                        k_f16=k.astype(np.float16).view(np.uint16),
                        v_f16=v.astype(np.float16).view(np.uint16))

    L, G, D, cap = 36, 8, 128, 4
    np.savez_compressed(HERE / "layout_selfcheck.npz", layers=L, kv_heads=G, head_dim=D,
                        capacity=cap, front=0, back=L * cap * G * D - 1,
                        back_coord=np.array([L - 1, 3, G - 1, D - 1]))

    past = 40
    n_past = past * G * D
    j = np.arange(n_past)
    past_k = ((j % 31 - 15) / 31.0).astype(np.float32).reshape(past, G, D)
    past_v = ((j % 29 - 14) / 29.0).astype(np.float32).reshape(past, G, D)
    s = np.arange(G * D)
    new_k = ((s % 23 - 11) / 23.0).astype(np.float32).reshape(1, G, D)
    new_v = new_k.copy()
    qi = np.arange(32 * D)
    q = ((qi % 127 - 63) / 63.0).astype(np.float32).reshape(1, 32, D)
    k16_past, v16_past = cpu_oracle.append_rows(past_k, past_v, np.arange(past), cos, sin,
                                                rope=False)
    k16_new, v16_new = cpu_oracle.append_rows(new_k, new_v, np.array([past]), cos, sin,
                                              rope=True)
    k_cache = np.concatenate([k16_past, k16_new], 0)
    v_cache = np.concatenate([v16_past, v16_new], 0)
    q_roped = cpu_oracle.rope_neox(q[0], cos[past], sin[past])[None]
    out = cpu_oracle.decode_attn(q_roped, [k_cache], [v_cache], cpu_oracle.EXACT)
    np.savez_compressed(HERE / "decode_seed.npz", past_k=past_k, past_v=past_v, new_k=new_k,
                        new_v=new_v, q=q, pos=past, k_cache=k_cache, v_cache=v_cache,
                        out=out)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
