"""CUDA op parity: the reference's known-answer tests replayed on the device,
and every token-loop kernel against the oracle on seeded inputs.

Tolerances: the KATs use the reference tests' own tolerances. Random-input
comparisons use an fp32 dot-product bound: |gpu - ref| <= 8 * sqrt(n) *
2^-24 * sum|a_i b_i| (+ a tiny absolute floor), since the kernels sum in a
different order than the reference's 16-lane NEON accumulation.
"""
import math

import numpy as np
import pytest
import torch

import kat_cases as K
from minfer_b200.gguf_synth import cast_weights
from oracle.oracle_py import PortOps

pytestmark = pytest.mark.gpu

EPS32 = 2.0 ** -24


def dot_tol(absprod_sum: np.ndarray, n: int) -> np.ndarray:
    return 8.0 * math.sqrt(n) * EPS32 * absprod_sum + 1e-7


def T(a, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.to(dev)


@pytest.fixture(scope="module")
def ops(gpu):
    from minfer_b200 import ops as o

    return o


@pytest.fixture(scope="module")
def orc():
    return PortOps()


def widen(w: np.ndarray, dt: int) -> np.ndarray:
    if dt == 0:
        return w.astype(np.float64)
    if dt == 1:
        return w.view(np.float16).astype(np.float64)
    return (w.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


DT_NAME = {0: "f32", 1: "f16", 2: "bf16"}


# ------------------------------------------------------------------ KATs

def test_kat_matmul(ops, gpu):
    for name, x, w, off, d_out, d_in, exp, tol in K.matmul_cases():
        out = torch.zeros(d_out, device=gpu)
        ops.matmul(out, T(x, gpu), T(w, gpu), off, d_out, d_in)
        np.testing.assert_allclose(out.cpu().numpy(), exp, atol=tol, rtol=0, err_msg=name)
    for name, dt, bits, x, off, d_out, d_in, exp, tol in K.matmul_16bit_cases():
        out = torch.zeros(d_out, device=gpu)
        ops.matmul(out, T(x, gpu), T(bits.view(np.int16), gpu), off, d_out, d_in, dtype=DT_NAME[dt])
        np.testing.assert_allclose(out.cpu().numpy(), exp, atol=tol, rtol=0, err_msg=name)


def test_kat_matmul_offset(ops, gpu):
    x, w32, w16, wbf, off, d_out, d_in = K.offset_case()
    res = []
    for w, dt in ((w32, "f32"), (w16.view(np.int16), "f16"), (wbf.view(np.int16), "bf16")):
        out = torch.zeros(d_out, device=gpu)
        ops.matmul(out, T(x, gpu), T(w, gpu), off, d_out, d_in, dtype=dt)
        res.append(out.cpu().numpy())
    np.testing.assert_allclose(res[1], res[0], atol=1e-6, rtol=0)
    np.testing.assert_allclose(res[2], res[0], atol=1e-6, rtol=0)
    np.testing.assert_allclose(res[0], np.full(d_out, 136.0, np.float32), atol=1e-6)  # expert 2: +1 weights


def test_kat_rmsnorm(ops, gpu):
    for name, x, w, eps, exp, tol in K.rmsnorm_cases():
        out = torch.zeros(x.size, device=gpu)
        ops.rmsnorm(out, T(x, gpu), T(w, gpu), x.size, eps)
        np.testing.assert_allclose(out.cpu().numpy(), exp, atol=tol, rtol=0, err_msg=name)


def test_kat_rope(ops, gpu):
    for name, neox, x, d_head, d_rot, pos, exp, tol in K.rope_cases():
        out = torch.zeros(x.size, device=gpu)
        fn = ops.neox_rope if neox else ops.il_rope
        fn(out, T(x, gpu), 0, d_head, d_rot, 10000.0, pos)
        np.testing.assert_allclose(out.cpu().numpy(), exp, atol=tol, rtol=0, err_msg=name)
    for name, neox in K.rope_partial_cases():
        x = torch.ones(6, device=gpu)
        out = torch.ones(6, device=gpu)
        (ops.neox_rope if neox else ops.il_rope)(out, x, 0, 6, 4, 10000.0, 1)
        o = out.cpu().numpy()
        assert o[0] != 1.0 or o[1 if not neox else 2] != 1.0
        assert o[4] == 1.0 and o[5] == 1.0
    # in place at position 0 is the identity (test_rope.cpp:128-145)
    for neox in (False, True):
        d = torch.tensor([1.0, 2.0, 3.0, 4.0], device=gpu)
        (ops.neox_rope if neox else ops.il_rope)(d, d, 0, 4, 4, 10000.0, 0)
        np.testing.assert_allclose(d.cpu().numpy(), [1, 2, 3, 4], atol=1e-6)


def test_kat_attn(ops, gpu):
    q, k, v, seq, dh, kvd, w, exp, tol = K.attn_weights_case()
    sc = torch.zeros(seq, device=gpu)
    out = torch.zeros(dh, device=gpu)
    ops.attn(sc, out, T(q, gpu), T(k, gpu), T(v, gpu), seq, dh, kvd)
    np.testing.assert_allclose(sc.cpu().numpy(), w, atol=tol)
    np.testing.assert_allclose(out.cpu().numpy(), exp, atol=tol)
    # single position (test_attn.cpp:9-24)
    sc = torch.zeros(1, device=gpu)
    out = torch.zeros(4, device=gpu)
    ops.attn(sc, out, T(np.array([1, 0, 0, 0], np.float32), gpu), T(np.array([1, 0, 0, 0], np.float32), gpu),
             T(np.array([2, 3, 4, 5], np.float32), gpu), 1, 4, 4)
    np.testing.assert_allclose(out.cpu().numpy(), [2, 3, 4, 5], atol=1e-6)
    assert abs(sc.item() - 1.0) < 1e-6
    # dominated output (test_attn.cpp:88-110 of the reference's last case)
    sc = torch.zeros(2, device=gpu)
    out = torch.zeros(2, device=gpu)
    ops.attn(sc, out, T(np.array([1, 0], np.float32), gpu), T(np.array([1000, 0, 0, 0], np.float32), gpu),
             T(np.array([5, 7, 100, 200], np.float32), gpu), 2, 2, 2)
    o = out.cpu().numpy()
    assert abs(o[0] - 5) < 0.1 and abs(o[1] - 7) < 0.1


def test_kat_route(ops, gpu):
    for name, x, w, n_exp, k, exp_ids, check in K.route_cases():
        ids = torch.zeros(k, dtype=torch.int32, device=gpu)
        wts = torch.zeros(k, device=gpu)
        scores = torch.zeros(n_exp, device=gpu)
        ops.route(T(x, gpu), ids, wts, scores, T(w.ravel(), gpu), 16, n_exp, k)
        assert ids.cpu().tolist() == exp_ids, name
        wv = wts.cpu().numpy()
        if k == 1:
            assert abs(wv[0] - 1.0) < 1e-6
        if check == "normalised":
            assert abs(wv.sum() - 1.0) < 1e-6 and wv[0] > wv[1]
        if check == "descending":
            assert all(wv[i] >= wv[i + 1] for i in range(k - 1))


def test_kat_softmax_silu(ops, gpu):
    for name, x, exp, tol in K.softmax_cases():
        out = torch.zeros(x.size, device=gpu)
        ops.softmax(out, T(x, gpu), x.size)
        np.testing.assert_allclose(out.cpu().numpy(), exp, atol=tol, err_msg=name)
    out = torch.zeros(3, device=gpu)
    ops.softmax(out, T(np.array([1000, 1001, 999], np.float32), gpu), 3)
    o = out.cpu().numpy()
    assert np.isfinite(o).all() and o[1] > o[0] and o[1] > o[2]
    out = torch.zeros(5, device=gpu)
    ops.softmax(out, T(np.arange(1, 6, dtype=np.float32), gpu), 5)
    assert abs(out.sum().item() - 1.0) < 1e-6
    xs = np.array([c[0] for c in K.silu_cases()], np.float32)
    out = torch.zeros(xs.size, device=gpu)
    ops.silu(out, T(xs, gpu), xs.size)
    np.testing.assert_allclose(out.cpu().numpy(), [c[1] for c in K.silu_cases()], atol=1e-6)


# ------------------------------------------------------------------ GEMV family

SHAPES = [(16, 16), (37, 256), (1024, 1024), (1000, 768), (4096 + 2048, 4096), (512, 12288), (4096, 25600),
          (129, 5120)]


@pytest.mark.parametrize("dt", [0, 1, 2])
@pytest.mark.parametrize("shape", SHAPES)
def test_matmul_vs_oracle(ops, orc, gpu, dt, shape):
    d_out, d_in = shape
    if dt == 0 and d_out * d_in > 40_000_000:
        pytest.skip("fp32 case covered by the smaller shapes")
    rng = np.random.default_rng(d_out * 131 + d_in + dt)
    x = rng.standard_normal(d_in).astype(np.float32)
    w = cast_weights(rng.standard_normal(d_out * d_in).astype(np.float32) * 0.02, DT_NAME[dt])
    out = torch.zeros(d_out, device=gpu)
    wt = T(w.view(np.int16) if dt else w, gpu)
    ops.matmul(out, T(x, gpu), wt, 0, d_out, d_in, dtype=DT_NAME[dt])
    got = out.cpu().numpy()
    ref = orc.matmul(x, w, dt, 0, d_out, d_in)
    W = widen(w, dt).reshape(d_out, d_in)
    exact = W @ x.astype(np.float64)
    tol = dot_tol(np.abs(W) @ np.abs(x.astype(np.float64)), d_in)
    assert np.all(np.abs(got - exact) <= tol), np.max(np.abs(got - exact) / tol)
    assert np.all(np.abs(ref - exact) <= tol)


@pytest.mark.parametrize("dt", [0, 2])
def test_rmsnorm_matmul_and_residual(ops, orc, gpu, dt):
    rng = np.random.default_rng(7 + dt)
    d_in, d_out = 2048, 3072
    x = rng.standard_normal(d_in).astype(np.float32)
    nw = (1.0 + 0.1 * rng.standard_normal(d_in)).astype(np.float32)
    w = cast_weights(rng.standard_normal(d_out * d_in).astype(np.float32) * 0.02, DT_NAME[dt])
    wt = T(w.view(np.int16) if dt else w, gpu)
    y = torch.zeros(d_out, device=gpu)
    ops.rmsnorm_matmul(y, T(x, gpu), T(nw, gpu), 1e-6, wt, d_out, d_in, dtype=DT_NAME[dt])
    xn = orc.rmsnorm(x, nw, 1e-6)
    W = widen(w, dt).reshape(d_out, d_in)
    exact = W @ xn.astype(np.float64)
    tol = dot_tol(np.abs(W) @ np.abs(xn.astype(np.float64)), d_in) + 2e-6 * np.abs(exact)
    assert np.all(np.abs(y.cpu().numpy() - exact) <= tol)
    # residual: x2 += W2 a
    a = rng.standard_normal(d_out).astype(np.float32)
    w2 = cast_weights(rng.standard_normal(d_in * d_out).astype(np.float32) * 0.02, DT_NAME[dt])
    res = rng.standard_normal(d_in).astype(np.float32)
    rt = T(res, gpu)
    ops.matmul_residual(rt, T(a, gpu), T(w2.view(np.int16) if dt else w2, gpu), d_in, d_out, dtype=DT_NAME[dt])
    W2 = widen(w2, dt).reshape(d_in, d_out)
    exact = res.astype(np.float64) + W2 @ a.astype(np.float64)
    tol = dot_tol(np.abs(W2) @ np.abs(a.astype(np.float64)), d_out) + EPS32 * np.abs(exact)
    assert np.all(np.abs(rt.cpu().numpy() - exact) <= tol)


@pytest.mark.parametrize("dt", [0, 1, 2])
@pytest.mark.parametrize("d_out,d_in", [(4096, 12288), (5120, 25600), (1024, 3072), (3000, 8192)])
def test_matmul_residual_wide_rows(ops, gpu, dt, d_out, d_in):
    """The residual GEMV of the down projections (rows of 12-51 KB: split over
    a cluster of CTAs, partials reduced in distributed shared memory) against
    a float64 product, within an fp32 dot-product bound."""
    if dt == 0 and d_in > 8192:
        pytest.skip("fp32 case covered by the narrower shapes")
    rng = np.random.default_rng(d_out + d_in + dt)
    a = rng.standard_normal(d_in).astype(np.float32)
    w = cast_weights(rng.standard_normal(d_out * d_in).astype(np.float32) * 0.02, DT_NAME[dt])
    res = rng.standard_normal(d_out).astype(np.float32)
    rt = T(res, gpu)
    wt = T(w.view(np.int16) if dt else w, gpu)
    for rep in range(2):  # twice: the second call starts from the first result
        ops.matmul_residual(rt, T(a, gpu), wt, d_out, d_in, dtype=DT_NAME[dt])
    W = widen(w, dt).reshape(d_out, d_in)
    prod = W @ a.astype(np.float64)
    exact = res.astype(np.float64) + 2 * prod
    tol = 2 * dot_tol(np.abs(W) @ np.abs(a.astype(np.float64)), d_in) + 2 * EPS32 * np.abs(exact)
    got = rt.cpu().numpy()
    assert np.all(np.abs(got - exact) <= tol), np.max(np.abs(got - exact) / tol)


@pytest.mark.parametrize("dt", [0, 1, 2])
def test_swiglu(ops, orc, gpu, dt):
    rng = np.random.default_rng(11 + dt)
    d_in, F = 1024, 1536
    x = rng.standard_normal(d_in).astype(np.float32)
    nw = np.ones(d_in, np.float32)
    g = cast_weights(rng.standard_normal(F * d_in).astype(np.float32) * 0.02, DT_NAME[dt]).reshape(F, d_in)
    u = cast_weights(rng.standard_normal(F * d_in).astype(np.float32) * 0.02, DT_NAME[dt]).reshape(F, d_in)
    gu = np.empty((2 * F, d_in), dtype=g.dtype)
    gu[0::2] = g
    gu[1::2] = u
    h = torch.zeros(F, device=gpu)
    ops.swiglu_matmul(h, T(x, gpu), T(nw, gpu), 1e-6, T(gu.view(np.int16) if dt else gu, gpu), F, d_in,
                      dtype=DT_NAME[dt])
    xn = orc.rmsnorm(x, nw, 1e-6)
    gr = orc.matmul(xn, g.ravel(), dt, 0, F, d_in)
    ur = orc.matmul(xn, u.ravel(), dt, 0, F, d_in)
    ref = np.array([orc.silu(float(a)) for a in gr], np.float32) * ur
    np.testing.assert_allclose(h.cpu().numpy(), ref, rtol=2e-5, atol=2e-6)


def test_lm_head_argmax(ops, orc, gpu):
    rng = np.random.default_rng(5)
    V, d = 50000, 1024
    x = rng.standard_normal(d).astype(np.float32)
    nw = np.ones(d, np.float32)
    w = cast_weights(rng.standard_normal(V * d).astype(np.float32) * 0.02, "bf16")
    # plant an exact tie at the top between rows 40001 and 17 (same weights):
    # the first maximum (row 17) must win, as std::max_element
    w = w.reshape(V, d)
    w[17] = cast_weights(x * 0.5, "bf16")
    w[40001] = w[17]
    logits = torch.zeros(V, device=gpu)
    ws = torch.zeros(ops.lm_head_workspace_bytes() // 4 + 1, dtype=torch.int32, device=gpu)
    st = torch.zeros(8, dtype=torch.int32, device=gpu)
    wt = T(w.ravel().view(np.int16), gpu)
    for rep in range(3):  # the workspace counter must come back to zero each call
        ops.lm_head(logits, T(x, gpu), T(nw, gpu), 1e-6, wt, V, d, step_state=st, workspace=ws, dtype="bf16")
        lg = logits.cpu().numpy()
        assert st[2].item() == int(np.argmax(lg)) == 17
    xn = orc.rmsnorm(x, nw, 1e-6)
    ref = orc.matmul(xn, w.ravel(), 2, 0, V, d)
    np.testing.assert_allclose(lg, ref, rtol=0, atol=1e-4)
    assert ws[0].item() == 0


# ------------------------------------------------------------------ attention

def _attn_reference(orc, qkv, qn, kn, eps, rope, kc_hist, vc_hist, pos, H, Hkv, D):
    """Oracle path of module.cpp:193-234 for one layer (history rows given)."""
    q = qkv[:H * D].copy()
    k = qkv[H * D:(H + Hkv) * D].copy()
    v = qkv[(H + Hkv) * D:].copy()
    for h in range(H):
        q[h * D:(h + 1) * D] = orc.rmsnorm(q[h * D:(h + 1) * D], qn, eps)
        q = orc.rope(q, h, D, D, 1e6, pos, out=q)
    for h in range(Hkv):
        k[h * D:(h + 1) * D] = orc.rmsnorm(k[h * D:(h + 1) * D], kn, eps)
        k = orc.rope(k, h, D, D, 1e6, pos, out=k)
    K_ = np.concatenate([kc_hist[:pos], k.reshape(1, Hkv, D)], 0)  # [pos+1, Hkv, D]
    V_ = np.concatenate([vc_hist[:pos], v.reshape(1, Hkv, D)], 0)
    out = np.zeros(H * D, np.float32)
    G = H // Hkv
    for h in range(H):
        kvh = h // G
        _, o = orc.attn(q[h * D:(h + 1) * D], np.ascontiguousarray(K_[:, kvh, :]).ravel(),
                        np.ascontiguousarray(V_[:, kvh, :]).ravel(), pos + 1, D, D)
        out[h * D:(h + 1) * D] = o
    return out, k.reshape(Hkv, D), v.reshape(Hkv, D)


@pytest.mark.parametrize("H,Hkv", [(4, 2), (16, 2), (8, 8), (32, 4), (32, 8), (16, 1)])
@pytest.mark.parametrize("pos", [0, 15, 16, 17, 255, 256, 300, 2049])
@pytest.mark.parametrize("split", ["default", 1, 7])
def test_attn_decode(ops, orc, gpu, H, Hkv, pos, split):
    D, S = 128, 2100
    rng = np.random.default_rng(H * 1000 + pos)
    qkv = rng.standard_normal((H + 2 * Hkv) * D).astype(np.float32)
    qn = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    kc_hist = rng.standard_normal((S, Hkv, D)).astype(np.float32)
    vc_hist = rng.standard_normal((S, Hkv, D)).astype(np.float32)
    rope = ops.rope_table(S, D, 1e6)
    # device cache layout [Hkv][S][D]
    kc = T(np.ascontiguousarray(kc_hist.transpose(1, 0, 2)), gpu)
    vc = T(np.ascontiguousarray(vc_hist.transpose(1, 0, 2)), gpu)
    n_split = ops.attn_default_split(Hkv, S) if split == "default" else split
    ws = torch.zeros(ops.attn_workspace_bytes(H, Hkv, D, n_split) // 4 + 1, dtype=torch.int32, device=gpu)
    st = torch.tensor([0, pos, 0, 0, 0, 0, 0, 0], dtype=torch.int32, device=gpu)
    out = torch.zeros(H * D, device=gpu)
    for rep in range(2):
        ops.attn_decode(T(qkv, gpu), T(qn, gpu), T(kn, gpu), 1e-6, rope.to(gpu), kc, vc, S, st, out, H, Hkv, D,
                        n_split, ws)
    ref, kref, vref = _attn_reference(orc, qkv, qn, kn, 1e-6, rope, kc_hist, vc_hist, pos, H, Hkv, D)
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=2e-5, atol=2e-5)
    kcn = kc.cpu().numpy()
    np.testing.assert_allclose(kcn[:, pos, :], kref, rtol=2e-6, atol=2e-6)
    np.testing.assert_array_equal(vc.cpu().numpy()[:, pos, :], vref)
    # rows other than `pos` untouched
    untouched = np.delete(kcn, pos, axis=1)
    np.testing.assert_array_equal(untouched, np.delete(kc_hist.transpose(1, 0, 2), pos, axis=1))
    assert ws[:Hkv].abs().sum().item() == 0  # counters back to zero


@pytest.mark.parametrize("H,Hkv,pos", [(32, 8, 4095), (32, 8, 32767), (64, 8, 32767), (32, 4, 32767)])
def test_attn_decode_long_context(ops, orc, gpu, H, Hkv, pos):
    """Decode attention at the benchmarked contexts (the 8B shape at 4096, the
    32B shape at a full 32K cache, the 30B-A3B head layout) against the oracle."""
    D, S = 128, pos + 1
    rng = np.random.default_rng(H * 7 + pos)
    qkv = rng.standard_normal((H + 2 * Hkv) * D).astype(np.float32)
    qn = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    kc_hist = rng.standard_normal((S, Hkv, D), dtype=np.float32)
    vc_hist = rng.standard_normal((S, Hkv, D), dtype=np.float32)
    rope = ops.rope_table(S, D, 1e6)
    kc = T(np.ascontiguousarray(kc_hist.transpose(1, 0, 2)), gpu)
    vc = T(np.ascontiguousarray(vc_hist.transpose(1, 0, 2)), gpu)
    n_split = ops.attn_default_split(Hkv, S)
    ws = torch.zeros(ops.attn_workspace_bytes(H, Hkv, D, n_split) // 4 + 1, dtype=torch.int32, device=gpu)
    st = torch.tensor([0, pos, 0, 0, 0, 0, 0, 0], dtype=torch.int32, device=gpu)
    out = torch.zeros(H * D, device=gpu)
    ops.attn_decode(T(qkv, gpu), T(qn, gpu), T(kn, gpu), 1e-6, rope.to(gpu), kc, vc, S, st, out, H, Hkv, D, n_split, ws)
    ref, kref, vref = _attn_reference(orc, qkv, qn, kn, 1e-6, rope, kc_hist, vc_hist, pos, H, Hkv, D)
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=2e-5, atol=2e-5)
    np.testing.assert_allclose(kc[:, pos, :].cpu().numpy(), kref, rtol=2e-6, atol=2e-6)
    np.testing.assert_array_equal(vc[:, pos, :].cpu().numpy(), vref)
    assert ws[:Hkv].abs().sum().item() == 0


def _bf16(a: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 (round to nearest even) -> fp32."""
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16).float().numpy()


@pytest.mark.parametrize("H,Hkv,pos", [(32, 8, 4095), (32, 8, 32767), (64, 8, 300), (16, 1, 2049), (8, 8, 17),
                                       (32, 4, 32767)])
def test_attn_decode_bf16_cache(ops, orc, gpu, H, Hkv, pos):
    """Opt-in bf16 KV cache: the history rows as stored (bf16, widened exactly),
    the appended K/V row rounded to nearest even and used rounded. Compared
    with the oracle on those same values: the rounded k may differ from the
    oracle's by one bf16 step where the fp32 values differ in their last bits."""
    D, S = 128, pos + 1
    rng = np.random.default_rng(H * 11 + pos)
    qkv = rng.standard_normal((H + 2 * Hkv) * D).astype(np.float32)
    qn = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    kc_hist = _bf16(rng.standard_normal((S, Hkv, D), dtype=np.float32))
    vc_hist = _bf16(rng.standard_normal((S, Hkv, D), dtype=np.float32))
    rope = ops.rope_table(S, D, 1e6)
    kc = T(np.ascontiguousarray(kc_hist.transpose(1, 0, 2)), gpu).to(torch.bfloat16)
    vc = T(np.ascontiguousarray(vc_hist.transpose(1, 0, 2)), gpu).to(torch.bfloat16)
    n_split = ops.attn_default_split(Hkv, S)
    ws = torch.zeros(ops.attn_workspace_bytes(H, Hkv, D, n_split) // 4 + 1, dtype=torch.int32, device=gpu)
    st = torch.tensor([0, pos, 0, 0, 0, 0, 0, 0], dtype=torch.int32, device=gpu)
    out = torch.zeros(H * D, device=gpu)
    ops.attn_decode(T(qkv, gpu), T(qn, gpu), T(kn, gpu), 1e-6, rope.to(gpu), kc, vc, S, st, out, H, Hkv, D, n_split, ws)
    _, kref, vref = _attn_reference(orc, qkv, qn, kn, 1e-6, rope, kc_hist, vc_hist, pos, H, Hkv, D)
    krow = kc[:, pos, :].float().cpu().numpy()
    np.testing.assert_allclose(krow, _bf16(kref), rtol=2 ** -7, atol=0)
    np.testing.assert_array_equal(vc[:, pos, :].float().cpu().numpy(), _bf16(vref))
    # the oracle's attention over exactly the rows the cache holds (history + the stored row)
    kh, vh = kc_hist.copy(), vc_hist.copy()
    kh[pos], vh[pos] = krow, _bf16(vref)
    ref = np.zeros(H * D, np.float32)
    G = H // Hkv
    for h in range(H):
        qh = orc.rope(orc.rmsnorm(qkv[h * D:(h + 1) * D], qn, 1e-6), 0, D, D, 1e6, pos)
        kvh = h // G
        _, o = orc.attn(qh, np.ascontiguousarray(kh[:, kvh, :]).ravel(), np.ascontiguousarray(vh[:, kvh, :]).ravel(),
                        pos + 1, D, D)
        ref[h * D:(h + 1) * D] = o
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=2e-5, atol=2e-5)
    assert ws[:Hkv].abs().sum().item() == 0


def test_attn_decode_position_out_of_range(ops, gpu):
    # a step record whose position has no cache row: nothing is written, the output is zero
    D, S, H, Hkv = 128, 64, 8, 2
    rng = np.random.default_rng(1)
    kc = T(rng.standard_normal(Hkv * S * D).astype(np.float32), gpu)
    vc = T(rng.standard_normal(Hkv * S * D).astype(np.float32), gpu)
    k0, v0 = kc.clone(), vc.clone()
    qkv = T(rng.standard_normal((H + 2 * Hkv) * D).astype(np.float32), gpu)
    nw = torch.ones(D, device=gpu)
    rope = ops.rope_table(S, D, 1e6).to(gpu)
    n_split = ops.attn_default_split(Hkv, S)
    ws = torch.zeros(ops.attn_workspace_bytes(H, Hkv, D, n_split) // 4 + 1, dtype=torch.int32, device=gpu)
    for pos in (S, S + 1000, -1):
        st = torch.tensor([0, pos, 0, 0, 0, 0, 0, 0], dtype=torch.int32, device=gpu)
        out = torch.full((H * D,), 7.0, device=gpu)
        ops.attn_decode(qkv, nw, nw, 1e-6, rope, kc, vc, S, st, out, H, Hkv, D, n_split, ws)
        torch.cuda.synchronize()
        assert out.abs().sum().item() == 0
        assert torch.equal(kc, k0) and torch.equal(vc, v0)
    assert ws[:Hkv].abs().sum().item() == 0


# ------------------------------------------------------------------ MoE

@pytest.mark.parametrize("dt,E", [(2, 128), (1, 16), (0, 16)])
def test_router_topk_and_experts(ops, orc, gpu, dt, E):
    """Router + top-k, grouped gate/up + SiLU and grouped down + weighted
    residual at the 30B-A3B layer shape (d 2048, k 8 of E, d_ff 768) in each
    weight dtype (the TMA-fed grouped kernels)."""
    rng = np.random.default_rng(3)
    d, k, F = 2048, 8, 768
    name = DT_NAME[dt]
    x = rng.standard_normal(d).astype(np.float32)
    nw = np.ones(d, np.float32)
    wr = (rng.standard_normal(E * d) * 0.02).astype(np.float32)
    ids = torch.zeros(k, dtype=torch.int32, device=gpu)
    wts = torch.zeros(k, device=gpu)
    scores = torch.zeros(E, device=gpu)
    xt = T(x, gpu)
    ops.router_topk(ids, wts, scores, xt, T(nw, gpu), 1e-6, T(wr, gpu), d, E, k)
    xn = orc.rmsnorm(x, nw, 1e-6)
    rid, rw, rs = orc.route(xn, wr, E, k)
    s = np.sort(rs)[::-1]
    assert s[k - 1] - s[k] > 1e-4  # not a near-tie case
    assert ids.cpu().tolist() == rid.tolist()
    np.testing.assert_allclose(wts.cpu().numpy(), rw, rtol=1e-5, atol=1e-6)
    # grouped expert SwiGLU + weighted down projection with residual
    g = cast_weights(rng.standard_normal(E * F * d).astype(np.float32) * 0.02, name).reshape(E, F, d)
    u = cast_weights(rng.standard_normal(E * F * d).astype(np.float32) * 0.02, name).reshape(E, F, d)
    dn = cast_weights(rng.standard_normal(E * d * F).astype(np.float32) * 0.02, name).reshape(E, d, F)
    gu = np.empty((E, 2 * F, d), g.dtype)
    gu[:, 0::2] = g
    gu[:, 1::2] = u
    dev = (lambda a: T(a.view(np.int16), gpu)) if dt else (lambda a: T(a, gpu))
    gu_d, dn_d = dev(gu), dev(dn)
    h = torch.zeros(k * F, device=gpu)
    ops.moe_swiglu(h, xt, T(nw, gpu), 1e-6, gu_d, ids, k, F, d, dtype=name)
    hr = np.zeros((k, F), np.float32)
    for sidx, e in enumerate(rid):
        gr = orc.matmul(xn, g.ravel(), dt, e * F * d, F, d)
        ur = orc.matmul(xn, u.ravel(), dt, e * F * d, F, d)
        hr[sidx] = np.array([orc.silu(float(a)) for a in gr], np.float32) * ur
    np.testing.assert_allclose(h.cpu().numpy().reshape(k, F), hr, rtol=3e-5, atol=3e-6)
    res = rng.standard_normal(d).astype(np.float32)
    rt = T(res, gpu)
    ops.moe_down_residual(rt, T(hr.ravel(), gpu), dn_d, ids, T(rw, gpu), k, d, F, dtype=name)
    ref = res.copy()
    for sidx, e in enumerate(rid):
        o = orc.matmul(hr[sidx], dn.ravel(), dt, e * d * F, d, F)
        ref = (ref + o * rw[sidx]).astype(np.float32)
    np.testing.assert_allclose(rt.cpu().numpy(), ref, rtol=2e-5, atol=2e-6)
    # the same FFN as one launch chain (the down projection's copies start
    # during the gate/up kernel): identical results to the separate calls.
    # Inputs alternate between chains, so a down kernel that read the previous
    # chain's expert ids would give a different residual.
    nwt, wrt = T(nw, gpu), T(wr, gpu)
    inputs = [rng.standard_normal(d).astype(np.float32) for _ in range(4)]
    ids_ch, wts_ch, h_ch = torch.zeros_like(ids), torch.zeros_like(wts), torch.zeros(k * F, device=gpu)
    for xi in inputs:
        x_sep, h_sep = T(xi, gpu), torch.zeros(k * F, device=gpu)
        ops.router_topk(ids, wts, scores, x_sep, nwt, 1e-6, wrt, d, E, k)
        ops.moe_swiglu(h_sep, x_sep, nwt, 1e-6, gu_d, ids, k, F, d, dtype=name)
        ops.moe_down_residual(x_sep, h_sep, dn_d, ids, wts, k, d, F, dtype=name)
        x_ch = T(xi, gpu)
        ops.moe_ffn(x_ch, h_ch, nwt, 1e-6, wrt, gu_d, dn_d, scores, ids_ch, wts_ch, d, F, E, k, dtype=name)
        assert torch.equal(ids_ch, ids) and torch.equal(h_ch, h_sep) and torch.equal(x_ch, x_sep)


def test_embed(ops, orc, gpu):
    rng = np.random.default_rng(9)
    V, d = 300, 256
    for dt in (0, 1, 2):
        w = cast_weights(rng.standard_normal(V * d).astype(np.float32), DT_NAME[dt])
        out = torch.zeros(d, device=gpu)
        ops.embed(out, T(w.view(np.int16) if dt else w, gpu), 123, d, dtype=DT_NAME[dt])
        np.testing.assert_array_equal(out.cpu().numpy(), orc.embed(w, dt, 123, d))
        st = torch.tensor([77, 0, 0, 0, 0, 0, 0, 0], dtype=torch.int32, device=gpu)
        ops.embed_step(out, T(w.view(np.int16) if dt else w, gpu), V, d, st, dtype=DT_NAME[dt])
        np.testing.assert_array_equal(out.cpu().numpy(), orc.embed(w, dt, 77, d))


def test_rope_table_matches_oracle(ops, orc):
    tab = ops.rope_table(40, 128, 1e6).numpy()
    rng = np.random.default_rng(1)
    x = rng.standard_normal(128).astype(np.float32)
    for pos in (0, 1, 39):
        c, s = tab[pos, :, 0], tab[pos, :, 1]
        x0, x1 = x[:64], x[64:]
        # first product fused, as the reference's compiled code contracts it
        f64 = np.float64
        r0 = (c.astype(f64) * x0.astype(f64) - (s * x1).astype(f64)).astype(np.float32)
        r1 = (s.astype(f64) * x0.astype(f64) + (c * x1).astype(f64)).astype(np.float32)
        mine = np.concatenate([r0, r1])
        np.testing.assert_array_equal(mine, orc.rope(x, 0, 128, 128, 1e6, pos))


def test_error_status(ops, gpu):
    from minfer_b200._lib import MinferError

    out = torch.zeros(16, device=gpu)
    with pytest.raises(MinferError):
        ops.matmul(out, torch.zeros(15, device=gpu), torch.zeros(16 * 15, device=gpu), 0, 16, 15)  # d_in % 16


@pytest.mark.parametrize("n,k", [(151936, 20), (151936, 64), (100, 64), (1030, 20), (5000, 1)])
def test_topk_candidates(gpu, n, k):
    """Device top-k (the sampler's candidate list): same ids and logits as a sort,
    largest first, equal values by lower index; NaN never wins; two calls in a row."""
    import ctypes as C

    from minfer_b200 import ops as O
    from minfer_b200._lib import check, cuda_lib

    lib = cuda_lib()
    g = torch.Generator(device="cpu").manual_seed(n + k)
    x = torch.randn(n, generator=g)
    x[n // 3] = float("nan")
    x[7] = x[11] = x.max() + 1.0  # a tie at the top: index 7 first
    ws_bytes = lib.mf_topk_workspace_bytes(n, k)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=gpu)
    ids = torch.empty(k, dtype=torch.int32, device=gpu)
    vals = torch.empty(k, dtype=torch.float32, device=gpu)
    xd = x.to(gpu)
    key = torch.where(torch.isnan(x), torch.tensor(float("-inf")), x).double()
    order = sorted(range(n), key=lambda i: (-key[i].item(), i))[:k]
    for _ in range(2):
        check(lib.mf_topk(C.c_void_p(xd.data_ptr()), n, k, C.c_void_p(ids.data_ptr()), C.c_void_p(vals.data_ptr()),
                          C.c_void_p(ws.data_ptr()), ws_bytes, C.c_void_p(O._stream())))
        torch.cuda.synchronize()
        assert ids.cpu().tolist() == order
        assert torch.equal(vals.cpu(), x[order])
