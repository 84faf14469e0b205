"""The opt-in bf16 KV cache (the reference keeps fp32 KV).

Two comparisons per model:
* against the oracle emulating the option (appended K/V rows rounded to bf16,
  nearest even): the same tolerances as the fp32 cache against the plain
  oracle, except that a rounded K/V element may sit one bf16 step away where
  the fp32 values differ in their last bits;
* against the reference's fp32-KV oracle, at the option's own tolerance:
  the distance is the rounding's own effect (the emulation's distance to the
  reference, plus the usual logit tolerance) and, for dense models, within
  KV_BF16_TOL x max|logit| (the rounding alone moves the tiny dense models'
  logits by 0.2-0.3 % of their scale; a MoE router may pick another expert).
"""
import numpy as np
import pytest

from conftest import TINY, tiny_model
from oracle.oracle_py import PortModel

pytestmark = pytest.mark.gpu

KV_BF16_TOL = 1e-2  # max-abs logit difference vs the fp32-KV reference, relative to max|logit|


def logit_tol(dtype: str) -> float:
    return 1e-3 if dtype == "f32" else 2e-2


@pytest.fixture(scope="module")
def Model(gpu):
    from minfer_b200.model import Qwen3Model, RunParams

    return Qwen3Model, RunParams


@pytest.mark.parametrize("name", ["tiny-f32", "tiny-bf16", "tiny-moe", "tiny-gqa8"])
def test_token_frames_vs_oracle(Model, name):
    """Decode frames token by token: logits every step and every KV row."""
    from minfer_b200.model import random_prompt

    Qwen3Model, RunParams = Model
    cfg = TINY[name]
    path = tiny_model(name)
    P = 24
    prompt = random_prompt(P, cfg.vocab, 9)
    emu = PortModel(path, max_seq=P + 1, kv_bf16=True)
    ref = PortModel(path, max_seq=P + 1)
    m = Qwen3Model(path, RunParams(max_seq_len=P + 1), kv_dtype="bf16").set_device("cuda")
    worst_emu = worst_ref = intrinsic = scale = 0.0
    for i, t in enumerate(prompt):
        for o in (emu, ref):
            o.forward(int(t), i, True)
        m.forward(int(t), i, True, True)
        lg = m.logits()
        worst_emu = max(worst_emu, float(np.abs(lg - emu.logits()).max()))
        worst_ref = max(worst_ref, float(np.abs(lg - ref.logits()).max()))
        intrinsic = max(intrinsic, float(np.abs(emu.logits() - ref.logits()).max()))
        scale = max(scale, float(np.abs(ref.logits()).max()))
        assert m.argmax() == int(np.argmax(lg))
    print(f"{name}: vs emulation {worst_emu:.3g}, vs fp32-KV reference {worst_ref:.3g} "
          f"(the rounding's own effect {intrinsic:.3g}, scale {scale:.3g})")
    assert worst_emu <= logit_tol(cfg.dtype)
    # the distance to the fp32-KV reference is the rounding's own effect
    assert worst_ref <= intrinsic + logit_tol(cfg.dtype)
    if not cfg.moe:  # (a rounded row can flip a router's choice, which moves MoE logits further)
        assert worst_ref <= KV_BF16_TOL * scale
    kvd = cfg.n_kv_heads * cfg.d_head
    for layer in range(cfg.n_layers):
        k, v = m.kv(layer, P)
        ko, vo = emu.kv(layer, P, kvd)
        # every stored value is a bf16 number
        kb = k.view(np.uint32)
        assert not np.any(kb & 0xFFFF) and not np.any(v.view(np.uint32) & 0xFFFF)
        # layer 0: rows from identical inputs, at most one bf16 step apart; deeper
        # layers also carry the effect of such steps in the rows below (measured
        # <= 1e-3 on the tiny models)
        atol = 1e-6 if layer == 0 else 4e-3
        np.testing.assert_allclose(k, ko, rtol=2 ** -7, atol=atol)
        np.testing.assert_allclose(v, vo, rtol=2 ** -7, atol=atol)


@pytest.mark.parametrize("name", ["tiny-f32", "tiny-bf16", "tiny-tp8"])
def test_batched_prefill_and_greedy_vs_oracle(Model, name):
    """Batched prefill (tensor cores, bf16 K/V operands widened from the cache)
    and greedy decode under teacher forcing: margins against the emulation,
    ids identical outside tolerance events."""
    from minfer_b200.model import random_prompt

    Qwen3Model, RunParams = Model
    cfg = TINY[name]
    path = tiny_model(name)
    P, G = 40, 24
    prompt = random_prompt(P, cfg.vocab, 13)
    emu = PortModel(path, max_seq=P + G + 1, kv_bf16=True)
    ref_ids, ref_mg = emu.generate(prompt, G)
    m = Qwen3Model(path, RunParams(num_iters=G, max_seq_len=P + G + 1), kv_dtype="bf16").set_device("cuda")
    ids, mg, _ = m.generate(prompt, G, forced=ref_ids, margins=True)
    np.testing.assert_allclose(mg, ref_mg, atol=2 * logit_tol(cfg.dtype))
    for i, (a, b) in enumerate(zip(ids, ref_ids)):
        assert a == b or ref_mg[i] < 1e-3, f"step {i}: {a} vs {b}, margin {ref_mg[i]}"


def test_cache_bytes_and_dtype_checks(Model):
    """The option lowers the bytes a generate run reports reading (the KV part
    halves), and is refused for other dtypes or once the model is on the GPU."""
    from minfer_b200._lib import MF_BF16, MinferError, check

    Qwen3Model, RunParams = Model
    path = tiny_model("tiny-bf16")
    a = Qwen3Model(path, RunParams(max_seq_len=64)).set_device("cuda")
    b = Qwen3Model(path, RunParams(max_seq_len=64), kv_dtype="bf16").set_device("cuda")
    _, _, sa = a.generate([1, 2, 3], 8)
    _, _, sb = b.generate([1, 2, 3], 8)
    assert sb.bytes_read < sa.bytes_read
    with pytest.raises(ValueError):
        Qwen3Model(path, RunParams(max_seq_len=64), kv_dtype="f16")
    with pytest.raises(MinferError):
        check(a._lib.mf_model_set_kv_dtype(a._h, MF_BF16))
