"""Q4_K projections and the backbone decode step on the GPU against the oracle.

The weights are N(0, 0.02) matrices quantised to Q4_K by the repo's encoder
(hkv_q4k_quantize); the oracle decodes the same bytes.  Activations are
quantised to Q8_K on both sides, so a projection differs from the oracle
only in the order of its float sums: 1e-5 relative (per vector, against the
largest output).  The two-layer backbone run (prompts fed token by token,
then greedy steps of two slots) must equal, bit for bit, the same step
issued call by call, every call of which is checked against the oracle on
the GPU's own inputs.
"""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DEV = "cuda:0"
PROJ_TOL = 1e-5
EPS = 1e-6


def rel_err(a, b):
    a = np.asarray(a, np.float64).reshape(np.shape(b)[0], -1)
    b = np.asarray(b, np.float64).reshape(a.shape)
    return float(np.max(np.abs(a - b).max(1) / np.maximum(np.abs(b).max(1), 1e-30)))


def q4k_matrix(hkv, rows, cols, seed, scale=0.02):
    gen = torch.Generator(device=DEV)
    gen.manual_seed(seed)
    w = torch.randn((rows, cols), generator=gen, device=DEV) * scale
    blocks = torch.empty((rows, cols // 256 * 144), dtype=torch.uint8, device=DEV)
    hkv.q4k_quantize(w, rows, cols, blocks)
    return w, blocks


def vec(seed, shape, scale=1.0, offset=0.0):
    gen = torch.Generator(device=DEV)
    gen.manual_seed(seed)
    return torch.randn(shape, generator=gen, device=DEV) * scale + offset


def test_encoder_round_trip(hkv_lib, oracle):
    import hkv
    quants = pytest.importorskip("gguf.quants")
    import gguf
    w, b = q4k_matrix(hkv, 64, 2560, 1)
    torch.cuda.synchronize()
    bn = b.cpu().numpy()
    dec = oracle.q4k_dequant(bn, 2560)
    assert np.array_equal(dec, quants.dequantize(bn, gguf.GGMLQuantizationType.Q4_K))
    wn = w.cpu().numpy()
    assert np.sqrt(np.mean((dec - wn) ** 2)) < 0.12 * np.sqrt(np.mean(wn ** 2))


@pytest.mark.parametrize("rows,cols,n,use_norm,use_res,tc", [
    (2560, 4096, 1, False, True, False),    # o_proj + residual (a warp per row)
    (2560, 9728, 1, False, True, False),    # ffn_down + residual
    (8208, 2560, 1, True, False, False),    # output head after output_norm
    (4096, 2560, 3, True, False, False),    # several vectors: tensor cores
    (300, 2560, 9, False, True, False),     # rows not a multiple of 16, n > 8 (two vector groups)
    (2560, 4096, 1, False, True, True),     # o_proj, one vector on the tensor cores
    (2560, 9728, 1, False, True, True),     # ffn_down (rows in flight beside a 9728-wide image)
    (8208, 2560, 16, True, False, False),   # the output head at batch 16
    (4096, 2560, 2, True, False, False),
    (40, 256, 3, True, True, False),        # one block per row, one partial tile
    (1000, 512, 16, False, True, False),    # 16 vectors in one launch, residual
    (130, 16384, 5, False, False, False),   # the widest rows, CTAs without rows
    (2560, 9728, 13, False, True, False),   # down: 8 + 5 vectors (two groups, one launch)
    (2560, 4096, 17, False, True, False),   # o_proj: 16 + 1 vectors
    (2560, 9728, 17, False, True, False),   # down: 8 + 8 + 1 vectors
])
def test_gemv_matches_oracle(hkv_lib, oracle, rows, cols, n, use_norm, use_res, tc):
    import hkv
    _, b = q4k_matrix(hkv, rows, cols, 10 + rows + n)
    x = vec(20 + n, (n, cols))
    norm = vec(30, (cols,), 0.1, 1.0) if use_norm else None
    res = vec(40, (n, rows)) if use_res else None
    y = torch.full((n, rows), float("nan"), device=DEV)
    hkv.q4k_gemv(b, rows, cols, x, y, n=n, norm=norm, eps=EPS, residual=res, tensor_cores=tc)
    torch.cuda.synchronize()
    xn = x.cpu().numpy()
    if use_norm:
        xn = oracle.rms_norm_mul(xn, EPS, norm.cpu().numpy())
    ref = oracle.q4k_gemv(b.cpu().numpy(), rows, cols, xn)
    if use_res:
        ref = ref + res.cpu().numpy()
    got = y.cpu().numpy()
    assert np.all(np.isfinite(got))
    assert rel_err(got, ref) <= PROJ_TOL
    hkv.q4k_sync_check()  # no bounded wait gave up


def test_gemv_in_place_residual(hkv_lib, oracle):
    import hkv
    _, b = q4k_matrix(hkv, 2560, 4096, 5)
    x = vec(6, (1, 4096))
    h = vec(7, (1, 2560))
    h0 = h.cpu().numpy()
    hkv.q4k_gemv(b, 2560, 4096, x, h, residual=h)
    torch.cuda.synchronize()
    ref = oracle.q4k_gemv(b.cpu().numpy(), 2560, 4096, x.cpu().numpy()) + h0
    assert rel_err(h.cpu().numpy(), ref) <= PROJ_TOL


@pytest.mark.parametrize("n,tc", [(1, False), (2, False), (1, True), (8, False), (17, False)])
def test_swiglu_matches_oracle(hkv_lib, oracle, n, tc):
    import hkv
    _, bg = q4k_matrix(hkv, 9728, 2560, 50)
    _, bu = q4k_matrix(hkv, 9728, 2560, 51)
    x = vec(52, (n, 2560))
    norm = vec(53, (2560,), 0.1, 1.0)
    y = torch.full((n, 9728), float("nan"), device=DEV)
    hkv.q4k_gemv(bg, 9728, 2560, x, y, n=n, norm=norm, eps=EPS, w_up=bu, tensor_cores=tc)
    torch.cuda.synchronize()
    m = oracle.rms_norm_mul(x.cpu().numpy(), EPS, norm.cpu().numpy())
    ref = oracle.silu_mul(oracle.q4k_gemv(bg.cpu().numpy(), 9728, 2560, m),
                          oracle.q4k_gemv(bu.cpu().numpy(), 9728, 2560, m))
    assert rel_err(y.cpu().numpy(), ref) <= PROJ_TOL


@pytest.mark.parametrize("n,tc", [(1, False), (3, False), (1, True), (16, False)])
def test_qkv_head_norm_matches_oracle(hkv_lib, oracle, n, tc):
    import hkv
    _, bq = q4k_matrix(hkv, 4096, 2560, 60)
    _, bk = q4k_matrix(hkv, 1024, 2560, 61)
    _, bv = q4k_matrix(hkv, 1024, 2560, 62)
    x = vec(63, (n, 2560))
    norm = vec(64, (2560,), 0.1, 1.0)
    qn = vec(65, (128,), 0.1, 1.0)
    kn = vec(66, (128,), 0.1, 1.0)
    q = torch.full((n, 4096), float("nan"), device=DEV)
    k = torch.full((n, 1024), float("nan"), device=DEV)
    v = torch.full((n, 1024), float("nan"), device=DEV)
    hkv.q4k_qkv(bq, bk, bv, 2560, x, qn, kn, q, k, v, n=n, norm=norm, eps=EPS, tensor_cores=tc)
    torch.cuda.synchronize()
    xn = oracle.rms_norm_mul(x.cpu().numpy(), EPS, norm.cpu().numpy())
    rq = oracle.q4k_gemv(bq.cpu().numpy(), 4096, 2560, xn).reshape(n, 32, 128)
    rk = oracle.q4k_gemv(bk.cpu().numpy(), 1024, 2560, xn).reshape(n, 8, 128)
    rv = oracle.q4k_gemv(bv.cpu().numpy(), 1024, 2560, xn)
    rq = oracle.rms_norm_mul(rq, EPS, qn.cpu().numpy())
    rk = oracle.rms_norm_mul(rk, EPS, kn.cpu().numpy())
    assert rel_err(q.cpu().numpy().reshape(-1, 128), rq.reshape(-1, 128)) <= PROJ_TOL
    assert rel_err(k.cpu().numpy().reshape(-1, 128), rk.reshape(-1, 128)) <= PROJ_TOL
    assert rel_err(v.cpu().numpy(), rv) <= PROJ_TOL


@pytest.mark.parametrize("rows,cols,swiglu", [(2560, 4096, False), (9728, 2560, True),
                                             (2560, 9728, False)])
def test_tensor_core_results_do_not_depend_on_batch(hkv_lib, rows, cols, swiglu):
    """On the tensor cores a vector's result is the same bits alone (n = 1)
    or among 4 or 11 others (one and two vector groups): the tiles, block slices
    and summation order depend on the matrix shape only."""
    import hkv
    _, b = q4k_matrix(hkv, rows, cols, 70 + rows)
    bu = q4k_matrix(hkv, rows, cols, 71 + rows)[1] if swiglu else None
    norm = vec(72, (cols,), 0.1, 1.0) if swiglu else None
    x = vec(73, (12, cols))
    outs = {}
    for n in (1, 5, 12):
        y = torch.empty((n, rows), device=DEV)
        hkv.q4k_gemv(b, rows, cols, x[:n], y, n=n, norm=norm, eps=EPS, w_up=bu, tensor_cores=True)
        outs[n] = y
    torch.cuda.synchronize()
    assert torch.equal(outs[1][0], outs[5][0]) and torch.equal(outs[1][0], outs[12][0])
    assert torch.equal(outs[5], outs[12][:5])
    hkv.q4k_sync_check()


def test_gemv_rejects_bad_shapes(hkv_lib):
    import hkv
    x = torch.zeros((1, 2560), device=DEV)
    y = torch.zeros((1, 64), device=DEV)
    w = torch.zeros(64 * 10 * 144, dtype=torch.uint8, device=DEV)
    with pytest.raises(hkv.HkvError, match="multiple of 256"):
        hkv.q4k_gemv(w, 64, 2500, x, y)
    with pytest.raises(hkv.HkvError, match="aligned"):
        hkv.q4k_gemv(w, 64, 2560, x[:, 1:], y)
    with pytest.raises(hkv.HkvError, match="no residual"):
        hkv.q4k_gemv(w, 64, 2560, x, y, residual=y, w_up=w)


def backbone_weights(hkv, n_layers, text_vocab):
    """Device weights (Q4_K blocks and F32 norms) and their numpy copies."""
    dev, host = {}, {}
    seed = [100]

    def mat(name, rows, cols):
        seed[0] += 1
        _, b = q4k_matrix(hkv, rows, cols, seed[0])
        dev[name] = b

    def norm(name, size):
        seed[0] += 1
        dev[name] = vec(seed[0], (size,), 0.1, 1.0)

    for l in range(n_layers):
        p = f"blk.{l}."
        mat(p + "attn_q", 4096, 2560)
        mat(p + "attn_k", 1024, 2560)
        mat(p + "attn_v", 1024, 2560)
        mat(p + "attn_output", 2560, 4096)
        mat(p + "ffn_gate", 9728, 2560)
        mat(p + "ffn_up", 9728, 2560)
        mat(p + "ffn_down", 2560, 9728)
        norm(p + "attn_norm", 2560)
        norm(p + "ffn_norm", 2560)
        norm(p + "attn_q_norm", 128)
        norm(p + "attn_k_norm", 128)
    mat("token_embd", text_vocab, 2560)
    mat("a.token_embd", 8 * 1026, 2560)
    mat("a.output", 8 * 1026, 2560)
    norm("output_norm", 2560)
    torch.cuda.synchronize()
    for k, t in dev.items():
        host[k] = t.cpu().numpy()
    return dev, host


class SerialStep:
    """The backbone step issued as separate calls with a device sync between
    them, each checked against the oracle on the GPU's own inputs: q/k/v,
    o_proj, FFN and output head at PROJ_TOL, attention over the slot's GPU
    cache at ATTN_TOL (the engine's parity tolerance)."""

    ATTN_TOL = 2e-3

    def __init__(self, hkv, oracle, eng, dev, host, n_layers, tc):
        self.hkv, self.o, self.eng, self.dev, self.host, self.L = hkv, oracle, eng, dev, host, n_layers
        self.tc = tc  # the projection kernels of the backbone under test
        self.cos, self.sin = oracle.rope_table()

    def run(self, h, slots, want_logits):
        hkv, o, dev, host = self.hkv, self.o, self.dev, self.host
        n = h.shape[0]
        h = h.clone()
        q = torch.empty((n, 4096), device=DEV)
        k = torch.empty((n, 1024), device=DEV)
        v = torch.empty((n, 1024), device=DEV)
        attn = torch.empty((n, 4096), device=DEV)
        g = torch.empty((n, 9728), device=DEV)
        pos = [self.eng.length(s) for s in slots]
        stream = torch.cuda.current_stream().cuda_stream
        for l in range(self.L):
            p = f"blk.{l}."
            hn = h.cpu().numpy()
            hkv.q4k_qkv(dev[p + "attn_q"], dev[p + "attn_k"], dev[p + "attn_v"], 2560, h,
                        dev[p + "attn_q_norm"], dev[p + "attn_k_norm"], q, k, v, n=n,
                        norm=dev[p + "attn_norm"], eps=EPS, tensor_cores=self.tc)
            torch.cuda.synchronize()
            xn = o.rms_norm_mul(hn, EPS, host[p + "attn_norm"])
            rq = o.rms_norm_mul(o.q4k_gemv(host[p + "attn_q"], 4096, 2560, xn).reshape(n, 32, 128),
                                EPS, host[p + "attn_q_norm"])
            rk = o.rms_norm_mul(o.q4k_gemv(host[p + "attn_k"], 1024, 2560, xn).reshape(n, 8, 128),
                                EPS, host[p + "attn_k_norm"])
            rv = o.q4k_gemv(host[p + "attn_v"], 1024, 2560, xn)
            assert rel_err(q.cpu().numpy().reshape(-1, 128), rq.reshape(-1, 128)) <= PROJ_TOL
            assert rel_err(k.cpu().numpy().reshape(-1, 128), rk.reshape(-1, 128)) <= PROJ_TOL
            assert rel_err(v.cpu().numpy(), rv) <= PROJ_TOL
            self.eng.decode_step(l, slots, q, k, v, attn, stream)
            torch.cuda.synchronize()
            # attention over the rows the GPU holds, with its own q
            ks, vs = [], []
            for e, s in enumerate(slots):
                kb = torch.empty((pos[e] + 1, 8, 128), dtype=torch.int16, device=DEV)
                vb = torch.empty_like(kb)
                self.eng.gather(s, l, 0, pos[e] + 1, kb, vb, stream)
                torch.cuda.synchronize()
                ks.append(kb.cpu().numpy().view(np.uint16))
                vs.append(vb.cpu().numpy().view(np.uint16))
            qn = q.cpu().numpy().reshape(n, 32, 128)
            qr = np.stack([o.rope_neox(qn[e], self.cos[pos[e]], self.sin[pos[e]]) for e in range(n)])
            assert rel_err(attn.cpu().numpy(), o.decode_attn(qr, ks, vs)) <= self.ATTN_TOL
            # h += Wo attn; g = silu(Wg m) * (Wu m); h += Wd g
            an, hn = attn.cpu().numpy(), h.cpu().numpy()
            hkv.q4k_gemv(dev[p + "attn_output"], 2560, 4096, attn, h, n=n, residual=h,
                         tensor_cores=self.tc)
            torch.cuda.synchronize()
            ref = hn + o.q4k_gemv(host[p + "attn_output"], 2560, 4096, an)
            assert rel_err(h.cpu().numpy(), ref) <= PROJ_TOL
            hn = h.cpu().numpy()
            hkv.q4k_gemv(dev[p + "ffn_gate"], 9728, 2560, h, g, n=n, norm=dev[p + "ffn_norm"],
                         eps=EPS, w_up=dev[p + "ffn_up"], tensor_cores=self.tc)
            torch.cuda.synchronize()
            m = o.rms_norm_mul(hn, EPS, host[p + "ffn_norm"])
            ref = o.silu_mul(o.q4k_gemv(host[p + "ffn_gate"], 9728, 2560, m),
                             o.q4k_gemv(host[p + "ffn_up"], 9728, 2560, m))
            assert rel_err(g.cpu().numpy(), ref) <= PROJ_TOL
            gn = g.cpu().numpy()
            hkv.q4k_gemv(dev[p + "ffn_down"], 2560, 9728, g, h, n=n, residual=h,
                         tensor_cores=self.tc)
            torch.cuda.synchronize()
            ref = hn + o.q4k_gemv(host[p + "ffn_down"], 2560, 9728, gn)
            assert rel_err(h.cpu().numpy(), ref) <= PROJ_TOL
        self.eng.advance(slots, 1)
        logits = None
        if want_logits:
            logits = torch.empty((n, 8 * 1026), device=DEV)
            hkv.q4k_gemv(dev["a.output"], 8 * 1026, 2560, h, logits, n=n, norm=dev["output_norm"],
                         eps=EPS, tensor_cores=self.tc)
            torch.cuda.synchronize()
            ref = o.q4k_gemv(host["a.output"], 8 * 1026, 2560,
                             o.rms_norm_mul(h.cpu().numpy(), EPS, host["output_norm"]))
            assert rel_err(logits.cpu().numpy(), ref) <= PROJ_TOL
        return h, logits


def test_backbone_steps_match_oracle(hkv_lib, oracle):
    """hkv_backbone_decode is bit-identical to the same step issued call by
    call (SerialStep), whose every projection and attention is checked
    against the oracle on the GPU's own inputs.  (Comparing against an
    independently evolved oracle over many steps is not a parity test: a
    1-ulp F16 rounding difference in a KV row, amplified by the next layer's
    Q8_K requantisation, grows to ~1e-2 over a few layers.)"""
    import hkv
    n_layers, vocab = 2, 512
    dev, host = backbone_weights(hkv, n_layers, vocab)
    e_bb = hkv.Engine(n_layers=n_layers, n_pages=64, max_slots=2, device=0, shuffle_seed=3,
                      lib=hkv_lib)
    e_ser = hkv.Engine(n_layers=n_layers, n_pages=64, max_slots=2, device=0, shuffle_seed=4,
                       lib=hkv_lib)
    bb = hkv.Backbone(e_bb, dev, text_vocab=vocab, rms_eps=EPS, max_batch=2)
    # max_batch 2: the backbone runs every projection on the tensor cores
    ser = SerialStep(hkv, oracle, e_ser, dev, host, n_layers, tc=True)
    emb = oracle.BackboneOracle(host, n_layers, eps=EPS)
    stream = torch.cuda.current_stream().cuda_stream
    hidden = torch.as_tensor(hkv.DeviceArray(bb.hidden_ptr, (2, 2560)), device=DEV)
    logits = torch.as_tensor(hkv.DeviceArray(bb.logits_ptr, (2, 8 * 1026)), device=DEV)
    codes = torch.as_tensor(hkv.DeviceArray(bb.codes_ptr, (2, 8), "<i4"), device=DEV)
    slots_bb = [e_bb.acquire(64), e_bb.acquire(64)]
    slots_ser = [e_ser.acquire(64), e_ser.acquire(64)]
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, vocab, 9), rng.integers(0, vocab, 4)]
    # prompts, one slot and one token at a time (the one-vector kernels)
    for e, ids in enumerate(prompts):
        for t, tok in enumerate(ids):
            last = t == len(ids) - 1
            bb.embed_text([int(tok)], stream)
            torch.cuda.synchronize()
            h0 = hidden[:1].clone()
            assert np.array_equal(h0.cpu().numpy(), emb.embed_text([int(tok)]))
            bb.decode([slots_bb[e]], want_logits=last, stream=stream)
            h_ser, lg_ser = ser.run(h0, [slots_ser[e]], last)
            torch.cuda.synchronize()
            assert torch.equal(hidden[:1], h_ser)
            if last:
                assert torch.equal(logits[:1], lg_ser)
    # joint greedy steps of both slots (the several-vector kernels)
    for step in range(3):
        launches0 = bb.kernel_launches
        if step == 0:
            bb.embed_text([1, 2], stream)
        else:
            bb.embed_codes(2, None, stream)  # the codes of the last decode
        torch.cuda.synchronize()
        h0 = hidden.clone()
        if step > 0:
            assert np.array_equal(h0.cpu().numpy(), emb.embed_codes(prev_codes))
        bb.decode(slots_bb, stream=stream)
        # embedding + 4 projections x 2 layers + output head + argmax
        assert bb.kernel_launches - launches0 == 1 + 4 * n_layers + 2
        h_ser, lg_ser = ser.run(h0, slots_ser, True)
        torch.cuda.synchronize()
        assert torch.equal(hidden, h_ser), step
        assert torch.equal(logits, lg_ser), step
        prev_codes = codes.cpu().numpy().copy()
        lg = lg_ser.cpu().numpy().reshape(2, 8, 1026)
        assert np.array_equal(prev_codes, lg.argmax(-1))
    bb.sync_check(stream)
    e_bb.sync_check(stream)
    assert [e_bb.length(s) for s in slots_bb] == [len(p) + 3 for p in prompts]
    bb.close()
    e_bb.close()
    e_ser.close()


def test_backbone_rejects_bad_ids(hkv_lib):
    import hkv
    dev, _ = backbone_weights(hkv, 1, 64)
    eng = hkv.Engine(n_layers=1, n_pages=8, max_slots=1, device=0, lib=hkv_lib)
    bb = hkv.Backbone(eng, dev, text_vocab=64, rms_eps=EPS, max_batch=1)
    with pytest.raises(hkv.HkvRangeError, match="outside"):
        bb.embed_text([64])
    bad = torch.tensor([[0, 0, 0, 1026, 0, 0, 0, 0]], dtype=torch.int32, device=DEV)
    bb.embed_codes(1, bad)
    with pytest.raises(hkv.HkvError, match="outside the table"):
        bb.sync_check()
    bb.sync_check()  # the error word was cleared
    bb.close()
    eng.close()
