"""Token-loop parity at the workloads' own shapes: the CUDA runtime against
golden fixtures made by the reference's own CPU token loop
(tests/golden/make_config_golden.py) on the same seeded GGUF files, which are
regenerated here from their seeds.

  c0  Qwen3-0.6B-shaped fp32, all 28 layers, vocabulary 151936: 16-token
      prompt, 128 greedy ids
  c1  Qwen3-1.7B-shaped bf16, all 28 layers: 512-token prompt (batched
      tensor-core prefill), 64 ids sampled at T 0.7, top-k 20, top-p 0.9, seed 42
  c2  Qwen3-8B-shaped bf16, first 4 layers at full width, untied lm_head
  c3  Qwen3-30B-A3B-shaped MoE, first 4 layers: expert ids of every layer at
      every forward, bit-exact
  c4  Qwen3-32B-shaped bf16, first 2 layers at full width

Greedy ids must be identical; a step whose reference top-2 margin is below
MARGIN_TOL may flip (a tolerance event, reported) and the comparison goes on
under teacher forcing. Sampled ids must be identical unless the flip rule of
tests/sampling_rule.py explains the flip (the reference's draw r lies within
the logits' error of a cumulative-probability boundary); every flip prints
that distance. Logits (a sample of the vocabulary at a few steps): max-abs
<= 1e-3 for the fp32 model, 2e-2 for bf16 (relative to the reference's fp32
path).
"""
import json
import os
import sys
from pathlib import Path

import numpy as np
import pytest

from conftest import model_dir

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "tests" / "golden"))

from make_config_golden import CASES, case_file_name, case_shape  # noqa: E402
from minfer_b200.gguf_synth import ensure_gguf  # noqa: E402
from sampling_rule import check_sampled  # noqa: E402

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
MARGIN_TOL = 1e-4


def logit_tol(dtype: str) -> float:
    return 1e-3 if dtype == "f32" else 2e-2


def load_case(name: str):
    g = json.loads((GOLDEN / f"config_{name}.json").read_text())
    path = ensure_gguf(model_dir() / case_file_name(name), case_shape(CASES[name]))
    return g, path


@pytest.fixture(scope="module")
def mm(gpu):
    from minfer_b200 import model

    return model


def check_logit_samples(g, lg_rows, steps):
    tol = logit_tol(g["dtype"])
    worst = 0.0
    for smp in g["logit_samples"]:
        row = lg_rows[steps.index(smp["step"])]
        d = np.abs(row[np.array(smp["idx"])] - np.array(smp["val"], np.float32)).max()
        worst = max(worst, float(d))
        assert d <= tol, f"{g['case']} step {smp['step']}: logits differ by {d}"
    return worst


@pytest.mark.parametrize("name", ["c0", "c2", "c4"])
def test_greedy_at_workload_shape(mm, name):
    g, path = load_case(name)
    P, G = len(g["prompt"]), len(g["ids"])
    prompt = np.array(g["prompt"], np.uint32)
    ref = np.array(g["ids"], np.uint32)
    steps = [s["step"] for s in g["logit_samples"]]
    m = mm.Qwen3Model(path, mm.RunParams(num_iters=G, max_seq_len=P + G + 1)).set_device("cuda")
    ids, mg, _, lg = m.generate(prompt, G, forced=ref, margins=True, logits_at=steps)
    events = []
    for i in range(G):
        if ids[i] != ref[i]:
            assert g["margins"][i] < MARGIN_TOL, f"{name}: id {i} differs ({ids[i]} vs {ref[i]}), margin {g['margins'][i]}"
            events.append(i)
    np.testing.assert_allclose(mg, g["margins"], atol=logit_tol(g["dtype"]))
    worst = check_logit_samples(g, lg, steps)
    # free-running greedy (the device argmax feeds back) up to the first tolerance event
    m2 = mm.Qwen3Model(path, mm.RunParams(num_iters=G, max_seq_len=P + G + 1)).set_device("cuda")
    free, _, _ = m2.generate(prompt, G)
    first = events[0] if events else G
    assert list(free[:first]) == list(ref[:first])
    print(f"{name}: {G} ids, tolerance events {events}, logit max-abs {worst:.3g}, min margin {min(g['margins']):.3g}")
    m.close()
    m2.close()


def test_sampled_at_workload_shape(mm):
    """c1: 512-token prompt through the batched prefill, then 64 sampled ids
    (teacher-forced on the reference's, so both sides draw the same r)."""
    from oracle.oracle_py import uniform_draws

    g, path = load_case("c1")
    P, G = len(g["prompt"]), len(g["ids"])
    sp = g["sampler"]
    prompt = np.array(g["prompt"], np.uint32)
    ref = np.array(g["ids"], np.uint32)
    rp = mm.RunParams(num_iters=G, max_seq_len=P + G + 1, top_k=sp["top_k"], temp=sp["temp"], top_p=sp["top_p"],
                      min_p=sp["min_p"], seed=sp["seed"])
    m = mm.Qwen3Model(path, rp).set_device("cuda")
    steps = list(range(G))
    ids, _, _, lg = m.generate(prompt, G, forced=ref, logits_at=steps)
    assert len(set(ref.tolist())) > G // 2  # really sampling
    r = uniform_draws(sp["seed"], G)
    cands = [(c["ids"], c["logits"]) for c in g["candidates"]]
    flips = check_sampled(ids, ref, cands, lg, sp["top_k"], sp["temp"], sp["top_p"], sp["min_p"], r, "c1")
    worst = check_logit_samples(g, [lg[s["step"]] for s in g["logit_samples"]], [s["step"] for s in g["logit_samples"]])
    print(f"c1: {G} sampled ids, flips {flips}, logit max-abs {worst:.3g}")
    assert len(flips) <= 2
    m.close()


def test_device_sampling_at_workload_shape(mm, monkeypatch):
    """c1 free-running (no teacher forcing): the device-sampled chain gives the
    host loop's 64 ids; the agreement with the reference's free-running ids is
    printed (they may part at a flip the teacher-forced test above explains)."""
    g, path = load_case("c1")
    P, G = len(g["prompt"]), len(g["ids"])
    sp = g["sampler"]
    prompt = np.array(g["prompt"], np.uint32)
    rp = mm.RunParams(num_iters=G, max_seq_len=P + G + 2, top_k=sp["top_k"], temp=sp["temp"], top_p=sp["top_p"],
                      min_p=sp["min_p"], seed=sp["seed"])
    got = {}
    for mode in ("device", "host"):
        if mode == "host":
            monkeypatch.setenv("MF_DEVICE_SAMPLE", "0")
        m = mm.Qwen3Model(path, rp).set_device("cuda")
        ids, _, _ = m.generate(prompt, G)
        got[mode] = [int(v) for v in ids]
        m.close()
    assert got["device"] == got["host"]
    same = next((i for i, (a, b) in enumerate(zip(got["device"], g["ids"])) if a != b), G)
    print(f"c1 free-running: device == host for {G} ids; equal to the reference's for the first {same}")


def test_moe_expert_ids_at_workload_shape(mm):
    """c3: the 8 expert ids of every layer at every forward (prompt and decode,
    teacher-forced) are the reference's, bit-exact; greedy ids and logits as above."""
    g, path = load_case("c3")
    P, G = len(g["prompt"]), len(g["ids"])
    ref = np.array(g["ids"], np.uint32)
    m = mm.Qwen3Model(path, mm.RunParams(num_iters=G, max_seq_len=P + G + 1)).set_device("cuda")
    L = g["layers"]
    toks = list(g["prompt"]) + [int(t) for t in ref]
    mism = []
    got_ids = []
    for f in range(P + G):
        m.forward(toks[f], f, f >= P - 1, False)  # logits from the last prompt token on
        for layer in range(L):
            e, _ = m.experts(layer)
            if list(e) != g["experts"][f][layer]:
                mism.append((f, layer, list(e), g["experts"][f][layer]))
        if P - 1 <= f < P + G - 1:
            got_ids.append(m.argmax())  # greedy id of step f - (P - 1)
    assert not mism, f"expert ids differ: {mism[:4]}"
    for i, (a, b) in enumerate(zip(got_ids, ref)):
        if a != b:
            assert g["margins"][i] < MARGIN_TOL, f"c3: id {i} differs ({a} vs {b})"
    # logit samples through generate
    m2 = mm.Qwen3Model(path, mm.RunParams(num_iters=G, max_seq_len=P + G + 1)).set_device("cuda")
    steps = [s["step"] for s in g["logit_samples"]]
    _, _, _, lg = m2.generate(np.array(g["prompt"], np.uint32), G, forced=ref, logits_at=steps)
    worst = check_logit_samples(g, lg, steps)
    print(f"c3: {P + G} forwards x {L} layers of expert ids identical; logit max-abs {worst:.3g}")
    m.close()
    m2.close()


def test_moe_batched_prefill_at_workload_shape(mm):
    """c3 through the batched MoE prefill (fp32 router + top-k per token,
    grouped tcgen05 expert GEMMs): the 8 expert ids of every prompt token at
    every layer are the reference's, bit-exact; the logits after the prompt
    match the reference's sample."""
    g, path = load_case("c3")
    P = len(g["prompt"])
    m = mm.Qwen3Model(path, mm.RunParams(max_seq_len=P + 1)).set_device("cuda")
    assert m.prefill(np.array(g["prompt"], np.uint32), 0, True, True)
    mism = []
    for layer in range(g["layers"]):
        ids, _ = m.prefill_experts(layer, P)
        for f in range(P):
            if list(ids[f]) != g["experts"][f][layer]:
                mism.append((f, layer, list(ids[f]), g["experts"][f][layer]))
    assert not mism, f"expert ids differ: {mism[:4]}"
    lg = m.logits()
    worst = 0.0
    for smp in g["logit_samples"]:
        if smp["step"] == 0:  # the logits of the last prompt token
            worst = float(np.abs(lg[np.array(smp["idx"])] - np.array(smp["val"], np.float32)).max())
            assert worst <= logit_tol(g["dtype"]), f"c3 prefill logits differ by {worst}"
    print(f"c3 batched prefill: {P} tokens x {g['layers']} layers of expert ids identical; logits after the prompt "
          f"max-abs {worst}")
    m.close()

