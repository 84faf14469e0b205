"""Token-loop parity of the CUDA runtime against the oracle on seeded synthetic
GGUF models: greedy ids, sampled ids, MoE expert ids, KV cache, logits.

Ids must be bit-exact. A step whose top-2 logit margin (reference side) is
below MARGIN_TOL is a tolerance event (fp32 summation order can flip it); the
test then keeps comparing under teacher forcing (the runtime is fed the
oracle's ids) and reports the event instead of failing on it.
Logits: max-abs <= 1e-3 for fp32 weights, 2e-2 for bf16/fp16 (relative to the
oracle's fp32 path).
"""
import json
from pathlib import Path

import numpy as np
import pytest

from conftest import TINY, tiny_model
from oracle.oracle_py import PortModel

pytestmark = pytest.mark.gpu

MARGIN_TOL = 1e-4
GOLDEN = Path(__file__).resolve().parent / "golden"


def logit_tol(dtype: str) -> float:
    return 1e-3 if dtype == "f32" else 2e-2


def check_ids(got, ref, margins, what):
    events = []
    for i, (a, b) in enumerate(zip(got, ref)):
        if a != b:
            assert margins[i] < MARGIN_TOL, f"{what}: id mismatch at step {i} ({a} vs {b}), margin {margins[i]}"
            events.append(i)
    return events


@pytest.fixture(scope="module")
def Model(gpu):
    from minfer_b200.model import Qwen3Model, RunParams

    return Qwen3Model, RunParams


@pytest.mark.parametrize("name", list(TINY))
def test_greedy_vs_oracle(Model, name):
    Qwen3Model, RunParams = Model
    path = tiny_model(name)
    cfg = TINY[name]
    P, G = 12, 40
    from minfer_b200.model import random_prompt

    prompt = random_prompt(P, cfg.vocab, 30)
    orc = PortModel(path, max_seq=P + G + 1)
    ref_ids, ref_mg = orc.generate(prompt, G)
    m = Qwen3Model(path, RunParams(num_iters=G, max_seq_len=P + G + 1)).set_device("cuda")
    ids, mg, st = m.generate(prompt, G, forced=ref_ids, margins=True)
    ev = check_ids(ids, ref_ids, ref_mg, name)
    np.testing.assert_allclose(mg, ref_mg, atol=logit_tol(cfg.dtype))
    assert st.num_tokens_gen == G and len(ev) <= 1
    # free-running greedy (no forcing) agrees up to the first tolerance event
    m2 = Qwen3Model(path, RunParams(num_iters=G, max_seq_len=P + G + 1)).set_device("cuda")
    free, _, _ = m2.generate(prompt, G)
    first = ev[0] if ev else G
    assert list(free[:first]) == list(ref_ids[:first])


@pytest.mark.parametrize("name", ["tiny-f32", "tiny-bf16", "tiny-moe"])
def test_logits_and_kv_vs_oracle(Model, name):
    Qwen3Model, RunParams = Model
    path = tiny_model(name)
    cfg = TINY[name]
    P = 20
    from minfer_b200.model import random_prompt

    prompt = random_prompt(P, cfg.vocab, 7)
    orc = PortModel(path, max_seq=P + 1)
    m = Qwen3Model(path, RunParams(max_seq_len=P + 1)).set_device("cuda")
    kvd = cfg.n_kv_heads * cfg.d_head
    if cfg.moe:
        orc.record_experts(True)
    n_events = 0
    for i, t in enumerate(prompt):
        orc.forward(int(t), i, True)
        m.forward(int(t), i, True, True)
        lo, lg = orc.logits(), m.logits()
        assert np.max(np.abs(lo - lg)) <= logit_tol(cfg.dtype), f"step {i}: {np.max(np.abs(lo - lg))}"
        assert m.argmax() == int(np.argmax(lg))
        if cfg.moe:
            ref_ids, _ = orc.recorded_experts(cfg.n_active)
            for layer in range(cfg.n_layers):
                ids, w = m.experts(layer)
                if list(ids) != list(ref_ids[i * cfg.n_layers + layer]):
                    n_events += 1
    assert n_events == 0
    for layer in range(cfg.n_layers):
        k, v = m.kv(layer, P)
        ko, vo = orc.kv(layer, P, kvd)
        np.testing.assert_allclose(k, ko, rtol=1e-4, atol=1e-5)
        np.testing.assert_allclose(v, vo, rtol=1e-4, atol=1e-5)


def oracle_sampled(path, prompt, G, kw):
    """The oracle's sampled ids and, per step, its top_k + 1 largest logits."""
    from sampling_rule import top_candidates

    P = len(prompt)
    orc = PortModel(path, max_seq=P + G + 1, **kw)
    for i, t in enumerate(prompt):
        orc.forward(int(t), i, i == P - 1)
    for t in prompt:
        orc.add_token(int(t))
    ids, cands = [], []
    for g in range(G):
        lg = orc.logits()
        cands.append(top_candidates(lg, kw["top_k"] + 1))
        nxt = orc.sample(lg)
        ids.append(nxt)
        orc.add_token(nxt)
        orc.forward(nxt, P + g, True)
    return np.array(ids, np.uint32), cands


SAMPLED = dict(top_k=20, temp=0.7, top_p=0.9, seed=42)  # the sampled workload's settings


def test_sampled_vs_oracle(Model):
    """Temperature 0.7, top-k 20, top-p 0.9, seed 42: teacher-forced on the
    oracle's ids, every id equals the oracle's unless the flip rule
    (tests/sampling_rule.py) explains it by the logits' error."""
    from oracle.oracle_py import uniform_draws
    from sampling_rule import check_sampled

    Qwen3Model, RunParams = Model
    name = "tiny-bf16"
    path = tiny_model(name)
    cfg = TINY[name]
    P, G = 16, 48
    from minfer_b200.model import random_prompt

    prompt = random_prompt(P, cfg.vocab, 42)
    ref_ids, cands = oracle_sampled(path, prompt, G, SAMPLED)
    m = Qwen3Model(path, RunParams(num_iters=G, max_seq_len=P + G + 1, **SAMPLED)).set_device("cuda")
    ids, _, _, lg = m.generate(prompt, G, forced=ref_ids, logits_at=list(range(G)))
    flips = check_sampled(ids, ref_ids, cands, lg, 20, 0.7, 0.9, 0.0, uniform_draws(42, G), name)
    assert len(flips) <= 1, flips
    assert len(set(ref_ids.tolist())) > 1  # really sampling


def test_sampled_from_device_candidates(Model, monkeypatch):
    """Sampling without logits requested reads back only the device top-k
    list: the ids equal those of the whole-vocabulary readback, and the
    oracle's under the flip rule."""
    from oracle.oracle_py import uniform_draws
    from sampling_rule import check_sampled

    Qwen3Model, RunParams = Model
    name = "tiny-bf16"
    path = tiny_model(name)
    cfg = TINY[name]
    P, G = 16, 48
    from minfer_b200.model import random_prompt

    prompt = random_prompt(P, cfg.vocab, 42)
    ref_ids, cands = oracle_sampled(path, prompt, G, SAMPLED)
    runs = []
    for host in ("0", "1"):
        monkeypatch.setenv("MF_HOST_TOPK", host)
        m = Qwen3Model(path, RunParams(num_iters=G, max_seq_len=P + G + 1, **SAMPLED)).set_device("cuda")
        ids, _, _ = m.generate(prompt, G, forced=ref_ids)  # teacher-forced: one draw per oracle step
        runs.append(list(ids))
    assert runs[0] == runs[1]
    m = Qwen3Model(path, RunParams(num_iters=G, max_seq_len=P + G + 1, **SAMPLED)).set_device("cuda")
    _, _, _, lg = m.generate(prompt, G, forced=ref_ids, logits_at=list(range(G)))
    flips = check_sampled(runs[0], ref_ids, cands, lg, 20, 0.7, 0.9, 0.0, uniform_draws(42, G), name)
    assert len(flips) <= 1, flips


def test_chained_matches_host_loop(Model):
    Qwen3Model, RunParams = Model
    path = tiny_model("tiny-bf16")
    P, G = 8, 24
    from minfer_b200.model import random_prompt

    prompt = random_prompt(P, TINY["tiny-bf16"].vocab, 3)
    m = Qwen3Model(path, RunParams(num_iters=G, max_seq_len=P + G + 2)).set_device("cuda")
    ids, _, _ = m.generate(prompt, G)
    m2 = Qwen3Model(path, RunParams(num_iters=G, max_seq_len=P + G + 2)).set_device("cuda")
    for i, t in enumerate(prompt):
        m2.forward(int(t), i, i == P - 1, False)
    first = m2.argmax()
    assert first == ids[0]
    last = m2.decode_chained(first, P, G - 1)
    assert last == ids[G - 1]


def test_golden_fixtures(Model):
    """Runtime vs the reference's own CPU run (fixtures made by tests/golden/make_golden.py)."""
    Qwen3Model, RunParams = Model
    files = sorted(GOLDEN.glob("model_*.json"))
    assert files, "golden fixtures missing"
    for f in files:
        g = json.loads(f.read_text())
        cfg = TINY[g["model"]]
        path = tiny_model(g["model"])
        kw = g["sampler"]
        P, G = len(g["prompt"]), len(g["ids"])
        m = Qwen3Model(path, RunParams(num_iters=G, max_seq_len=P + G + 1, **kw)).set_device("cuda")
        ids, mg, _ = m.generate(np.array(g["prompt"], np.uint32), G, forced=np.array(g["ids"], np.uint32),
                                margins=True)
        check_ids(ids, g["ids"], g["margins"], f.name)
        np.testing.assert_allclose(mg, g["margins"], atol=logit_tol(cfg.dtype))


@pytest.mark.parametrize("name,kw", [("tiny-bf16", dict(top_k=20, temp=0.7, top_p=0.9, seed=42)),
                                     ("tiny-f32", dict(top_k=40, temp=1.2, top_p=0.95, min_p=0.05, seed=7)),
                                     ("tiny-moe", dict(top_k=8, temp=0.9, top_p=1.0, seed=3))])
def test_device_sampling_matches_host_loop(Model, monkeypatch, name, kw):
    """Free-running sampled generate: the device chain (top-k candidates,
    softmax / top-p / min-p / temperature and the draw in a kernel, the id fed
    to the next frame on the device) gives the host loop's ids, with the same
    random stream; a second run continues the stream identically."""
    Qwen3Model, RunParams = Model
    from minfer_b200.model import random_prompt

    cfg = TINY[name]
    path = tiny_model(name)
    P, G = 12, 40
    prompt = random_prompt(P, cfg.vocab, 17)
    runs = {}
    for mode in ("device", "host"):
        if mode == "host":
            monkeypatch.setenv("MF_DEVICE_SAMPLE", "0")
        m = Qwen3Model(path, RunParams(num_iters=G, max_seq_len=2 * (P + G) + 2, **kw)).set_device("cuda")
        first, _, st = m.generate(prompt, G)
        second, _, _ = m.generate(prompt, G)  # continues the random stream
        third, _, _ = m.generate(prompt[:5], G // 2)  # another length: the replayed frames serve it too
        assert st.num_tokens_gen == G
        runs[mode] = (list(first), list(second), list(third))
        m.close()
    assert runs["device"] == runs["host"], f"{name}: device {runs['device']} vs host {runs['host']}"
    assert runs["device"][0] != runs["device"][1]  # the stream moved on



def test_generate_text_vs_oracle(Model):
    """BaseModel::generate(std::string&): chat template -> tokenizer -> GPU
    token loop -> decoded text, on a model file with a byte-level vocabulary.
    The ids must be the oracle's greedy ids for the same encoded prompt (cut
    after the first EOS, which ends the loop), up to a tolerance event."""
    from conftest import TEXT_MODEL, text_model
    from minfer_b200.tokenizer import Qwen3Tokenizer

    Qwen3Model, RunParams = Model
    path = text_model()
    G = 48
    text = "Hello, world! It's 2 + 2 = 4; 世界\n"
    m = Qwen3Model(path, RunParams(num_iters=G, max_seq_len=256)).set_device("cuda")
    res = m.generate_text(text)
    tok = Qwen3Tokenizer.from_gguf(path)
    assert res.formatted == f"<|im_start|>user\n{text}<|im_end|>\n<|im_start|>assistant\n"
    assert res.prompt_ids == tok.encode(res.formatted)
    assert tok.decode(res.prompt_ids) == res.formatted.encode()
    orc = PortModel(path, max_seq=len(res.prompt_ids) + G + 1)
    ref_ids, ref_mg = orc.generate(np.array(res.prompt_ids, np.uint32), G)
    ref = [int(i) for i in ref_ids]
    if tok.eos_id in ref:
        cut = ref.index(tok.eos_id) + 1
        ref, ref_mg = ref[:cut], ref_mg[:cut]
    ev = check_ids(res.ids, ref, ref_mg, "tiny-text")
    first = ev[0] if ev else len(ref)
    assert res.ids[:first] == ref[:first]
    if not ev:
        assert res.ids == ref and res.stats.num_tokens_gen == len(ref)
    assert res.text == tok.decode(res.ids)
    assert TEXT_MODEL.vocab == m.vocab_size
