"""The oracle, pinned (CPU only).

1. The reference's known-answer tests (tests/kat_cases.py) pass on the oracle
   restatement and on the reference's own compiled ops.
2. The restatement is bit-exact with the reference's compiled CPU path on
   random operands and on whole tiny models (ids, margins, expert ids).
3. The restatement reproduces the committed golden fixtures, which were made
   by the reference's own CPU run.
"""
import json
import math
import tempfile
from pathlib import Path

import numpy as np
import pytest

import kat_cases as K
from conftest import TINY, tiny_model
from minfer_b200.gguf_synth import cast_weights, random_prompt
from oracle.oracle_py import PortModel, PortOps, RefOps, ref_available, run_reference

GOLDEN = Path(__file__).resolve().parent / "golden"

needs_ref = pytest.mark.skipif(not ref_available(), reason="reference build (oracle/_ref) not present")


def backends():
    out = [("port", PortOps())]
    if ref_available():
        out.append(("reference", RefOps()))
    return out


@pytest.mark.parametrize("name,ops", backends())
def test_kat_matmul(name, ops):
    for case, x, w, off, d_out, d_in, exp, tol in K.matmul_cases():
        np.testing.assert_allclose(ops.matmul(x, w, 0, off, d_out, d_in), exp, atol=tol, rtol=0, err_msg=case)
    for case, dt, bits, x, off, d_out, d_in, exp, tol in K.matmul_16bit_cases():
        np.testing.assert_allclose(ops.matmul(x, bits, dt, off, d_out, d_in), exp, atol=tol, err_msg=case)
    x, w32, w16, wbf, off, d_out, d_in = K.offset_case()
    r32 = ops.matmul(x, w32, 0, off, d_out, d_in)
    np.testing.assert_allclose(ops.matmul(x, w16, 1, off, d_out, d_in), r32, atol=1e-6)
    np.testing.assert_allclose(ops.matmul(x, wbf, 2, off, d_out, d_in), r32, atol=1e-6)


@pytest.mark.parametrize("name,ops", backends())
def test_kat_rmsnorm_rope_attn(name, ops):
    for case, x, w, eps, exp, tol in K.rmsnorm_cases():
        np.testing.assert_allclose(ops.rmsnorm(x, w, eps), exp, atol=tol, err_msg=case)
    for case, neox, x, d_head, d_rot, pos, exp, tol in K.rope_cases():
        np.testing.assert_allclose(ops.rope(x, 0, d_head, d_rot, 10000.0, pos, neox=neox), exp, atol=tol,
                                   err_msg=case)
    for case, neox in K.rope_partial_cases():
        out = ops.rope(np.ones(6, np.float32), 0, 6, 4, 10000.0, 1, neox=neox, out=np.ones(6, np.float32))
        assert out[4] == 1.0 and out[5] == 1.0 and (out[0] != 1.0 or out[2] != 1.0)
    q, k, v, seq, dh, kvd, w, exp, tol = K.attn_weights_case()
    sc, out = ops.attn(q, k, v, seq, dh, kvd)
    np.testing.assert_allclose(sc, w, atol=tol)
    np.testing.assert_allclose(out, exp, atol=tol)


@pytest.mark.parametrize("name,ops", backends())
def test_kat_route_softmax_silu(name, ops):
    for case, x, w, n_exp, k, exp_ids, check in K.route_cases():
        ids, wts, _ = ops.route(x, w.ravel(), n_exp, k)
        assert ids.tolist() == exp_ids, case
        if check == "normalised":
            assert abs(wts.sum() - 1) < 1e-6 and wts[0] > wts[1]
    for case, x, exp, tol in K.softmax_cases():
        np.testing.assert_allclose(ops.softmax(x), exp, atol=tol, err_msg=case)
    for x, exp, tol in K.silu_cases():
        assert abs(ops.silu(x) - exp) < tol


@needs_ref
@pytest.mark.parametrize("dt", [0, 1, 2])
def test_restatement_bit_exact_ops(dt):
    po, ro = PortOps(), RefOps()
    rng = np.random.default_rng(dt)
    for d_out, d_in in ((37, 256), (300, 1024), (64, 2048)):
        x = rng.standard_normal(d_in).astype(np.float32)
        w = cast_weights(rng.standard_normal(d_out * d_in).astype(np.float32) * 0.02, {0: "f32", 1: "f16", 2: "bf16"}[dt])
        assert np.array_equal(po.matmul(x, w, dt, 0, d_out, d_in), ro.matmul(x, w, dt, 0, d_out, d_in))
        assert np.array_equal(po.embed(w, dt, 3, d_in), ro.embed(w, dt, 3, d_in))
    x = rng.standard_normal(128).astype(np.float32)
    for pos in (0, 1, 77, 4095, 32768):
        assert np.array_equal(po.rope(x, 0, 128, 128, 1e6, pos), ro.rope(x, 0, 128, 128, 1e6, pos))
        assert np.array_equal(po.rope(x, 0, 128, 128, 1e6, pos, neox=False), ro.rope(x, 0, 128, 128, 1e6, pos, neox=False))
    w = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    assert np.array_equal(po.rmsnorm(x, w, 1e-6), ro.rmsnorm(x, w, 1e-6))
    k = rng.standard_normal(128 * 33).astype(np.float32)
    v = rng.standard_normal(128 * 33).astype(np.float32)
    for a, b in zip(po.attn(x, k, v, 33, 128, 128), ro.attn(x, k, v, 33, 128, 128)):
        assert np.array_equal(a, b)
    xr = rng.standard_normal(256).astype(np.float32)
    wr = rng.standard_normal(16 * 256).astype(np.float32)
    for a, b in zip(po.route(xr, wr, 16, 4), ro.route(xr, wr, 16, 4)):
        assert np.array_equal(a, b)


@needs_ref
@pytest.mark.parametrize("name", ["tiny-bf16", "tiny-f32", "tiny-moe", "tiny-gqa8"])
def test_restatement_bit_exact_models(name):
    path = tiny_model(name)
    cfg = TINY[name]
    P, G = 10, 16
    with tempfile.TemporaryDirectory() as td:
        ref = run_reference(path, f"{td}/r", random_prompt=P, prompt_seed=5, gen=G, max_seq=P + G + 1)
    prompt = random_prompt(P, cfg.vocab, 5)
    assert ref["prompt"] == [int(t) for t in prompt]  # prompt draw restated exactly
    pm = PortModel(path, max_seq=P + G + 1)
    if cfg.moe:
        pm.record_experts(True)
    ids, mg = pm.generate(prompt, G)
    assert ids.tolist() == ref["ids"]
    assert np.array_equal(mg, np.array(ref["margins"], np.float32))
    if cfg.moe:
        e, _ = pm.recorded_experts(cfg.n_active)
        assert np.array_equal(e.reshape(ref["experts"].shape), ref["experts"])


@needs_ref
def test_restatement_bit_exact_sampled():
    path = tiny_model("tiny-bf16")
    P, G = 8, 24
    kw = dict(temp=0.7, top_k=20, top_p=0.9, seed=42)
    with tempfile.TemporaryDirectory() as td:
        ref = run_reference(path, f"{td}/r", random_prompt=P, prompt_seed=42, gen=G, max_seq=P + G + 1, **kw)
    pm = PortModel(path, max_seq=P + G + 1, top_k=20, temp=0.7, top_p=0.9, seed=42)
    ids, _ = pm.generate(random_prompt(P, 1024, 42), G)
    assert ids.tolist() == ref["ids"]


@pytest.mark.parametrize("fixture", sorted(p.name for p in GOLDEN.glob("model_*.json")))
def test_restatement_reproduces_golden(fixture):
    g = json.loads((GOLDEN / fixture).read_text())
    cfg = TINY[g["model"]]
    P, G = len(g["prompt"]), len(g["ids"])
    smp = g["sampler"]
    pm = PortModel(tiny_model(g["model"]), max_seq=P + G + 1, top_k=smp["top_k"], temp=smp["temp"],
                   top_p=smp["top_p"], seed=smp["seed"])
    if cfg.moe:
        pm.record_experts(True)
    ids, mg = pm.generate(np.array(g["prompt"], np.uint32), G)
    assert ids.tolist() == g["ids"]
    assert np.array_equal(mg, np.array(g["margins"], np.float32))
    if cfg.moe:
        e, _ = pm.recorded_experts(cfg.n_active)
        assert e.reshape(-1).tolist() == np.array(g["experts"]).reshape(-1).tolist()


def test_golden_logits_step0():
    g = json.loads((GOLDEN / "model_tiny-f32_greedy.json").read_text())
    P = len(g["prompt"])
    pm = PortModel(tiny_model("tiny-f32"), max_seq=P + 2)
    for i, t in enumerate(g["prompt"]):
        pm.forward(t, i, i == P - 1)
    assert np.array_equal(pm.logits(), np.array(g["logits_step0"], np.float32))


def test_tolerances_sane():
    # the parity tests' fp32 dot bound is loose enough for a 16-lane vs CTA-wide sum
    assert 8 * math.sqrt(4096) * 2.0 ** -24 < 1e-4


def test_kv_bf16_emulation_rounds_to_nearest_even():
    """The oracle's emulation of the runtime's opt-in bf16 KV cache: the first
    token's layer-0 K/V rows are the fp32 run's rows rounded to bf16, nearest
    even (numpy bit arithmetic as the check); later rows differ because the
    attention then reads rounded history."""
    cfg = TINY["tiny-bf16"]
    path = tiny_model("tiny-bf16")
    kvd = cfg.n_kv_heads * cfg.d_head
    a = PortModel(path, max_seq=4)
    b = PortModel(path, max_seq=4, kv_bf16=True)
    for m in (a, b):
        m.forward(5, 0, True)
    k32, v32 = a.kv(0, 1, kvd)
    k16, v16 = b.kv(0, 1, kvd)

    def rne(x):
        u = x.view(np.uint32).astype(np.uint64)
        u = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
        return u.view(np.float32)

    assert np.array_equal(k16, rne(k32)) and np.array_equal(v16, rne(v32))
    assert not np.array_equal(k16, k32)
    assert np.abs(b.logits() - a.logits()).max() > 0
