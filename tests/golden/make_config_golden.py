"""Golden fixtures at the workloads' own shapes, made by the reference's own
CPU token loop (oracle/_ref/minfer_ref_run, the reference sources compiled by
oracle/Makefile) on the seeded synthetic GGUF files.

Cases (the five workload models; the three large ones as depth-reduced
prefixes at full width and the real vocabulary, Qwen3Shape.prefix):
  c0  Qwen3-0.6B-shaped fp32, all 28 layers, 16-token prompt, 128 greedy ids
  c1  Qwen3-1.7B-shaped bf16, all 28 layers, 512-token prompt, 64 ids sampled
      at temperature 0.7, top-k 20, top-p 0.9, seed 42
  c2  Qwen3-8B-shaped bf16, first 4 of 36 layers, 32-token prompt, 32 greedy ids
  c3  Qwen3-30B-A3B-shaped MoE bf16, first 4 of 48 layers, 32 + 32 tokens,
      the 8 expert ids of every layer at every forward
  c4  Qwen3-32B-shaped bf16, first 2 of 64 layers, 32 + 32 tokens
Prompt ids: random_prompt(P, vocab, model seed), as BaseModel::benchmark
draws them (src/base/model.cpp:189-193).

Each fixture holds the ids, the top-2 logit margin of every step, and for a
few steps a sample of the logits: the 32 largest and 256 fixed random
vocabulary entries. The sampled case also holds, for every step, the
reference's 21 largest logits (the top-k list plus the next one) so a test
can rebuild the reference's sampling distribution.

Usage (needs oracle/_ref; writes tests/golden/config_<case>.json; the model
files go to $MF_MODEL_DIR or /dev/shm/minfer_b200_cfg):
    python tests/golden/make_config_golden.py [c0 c1 c2 c3 c4]
"""
from __future__ import annotations

import json
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from minfer_b200.gguf_synth import CONFIGS, ensure_gguf, random_prompt  # noqa: E402
from oracle import oracle_py  # noqa: E402

N_TOP, N_RANDOM, N_CAND = 32, 256, 21

CASES = {
    "c0": dict(model="qwen3-0.6b-f32", layers=None, prompt=16, gen=128, logit_steps=[0, 64, 127]),
    "c1": dict(model="qwen3-1.7b-bf16", layers=None, prompt=512, gen=64, logit_steps=[0, 32, 63],
               sampler=dict(temp=0.7, top_k=20, top_p=0.9, min_p=0.0, pres=0.0, seed=42)),
    "c2": dict(model="qwen3-8b-bf16", layers=4, prompt=32, gen=32, logit_steps=[0, 31]),
    "c3": dict(model="qwen3-30b-a3b-bf16", layers=4, prompt=32, gen=32, logit_steps=[0, 31], experts=True),
    "c4": dict(model="qwen3-32b-bf16", layers=2, prompt=32, gen=32, logit_steps=[0, 31]),
}


def case_shape(case: dict):
    shape = CONFIGS[case["model"]]
    return shape.prefix(case["layers"]) if case["layers"] else shape


def case_file_name(name: str) -> str:
    case = CASES[name]
    depth = f"-{case['layers']}l" if case["layers"] else ""
    return f"{case['model']}{depth}.gguf"


def logit_sample_indices(vocab: int, step: int) -> np.ndarray:
    """The fixed random vocabulary entries sampled at `step`."""
    return np.sort(np.random.default_rng(1000 + step).choice(vocab, N_RANDOM, replace=False))


def make(name: str, model_dir: Path) -> dict:
    case = CASES[name]
    shape = case_shape(case)
    path = ensure_gguf(model_dir / case_file_name(name), shape)
    prompt = random_prompt(case["prompt"], shape.vocab, shape.seed)
    smp = case.get("sampler", dict(temp=0.0, top_k=1, top_p=1.0, min_p=0.0, pres=0.0, seed=0))
    sampled = smp["temp"] > 0
    dump = [-1] if sampled else case["logit_steps"]
    with tempfile.TemporaryDirectory() as td:
        res = oracle_py.run_reference(path, f"{td}/r", prompt=prompt, gen=case["gen"],
                                      max_seq=case["prompt"] + case["gen"] + 1, dump_logits=dump,
                                      temp=smp["temp"], top_k=smp["top_k"], top_p=smp["top_p"],
                                      min_p=smp["min_p"], pres=smp["pres"], seed=smp["seed"],
                                      threads=os.cpu_count())
    lg = res["logits"]
    rows = {s: lg[i] for i, s in enumerate(range(case["gen"]) if sampled else case["logit_steps"])}
    out = {
        "case": name, "model": case["model"], "layers": shape.n_layers, "full_layers": CONFIGS[case["model"]].n_layers,
        "dtype": shape.dtype, "vocab": shape.vocab, "prompt_seed": shape.seed, "prompt": [int(t) for t in prompt],
        "sampler": smp, "ids": [int(v) for v in res["ids"]], "margins": [float(v) for v in res["margins"]],
        "logit_samples": [],
        "made_by": "oracle/_ref/minfer_ref_run (the reference's CPU token loop), tests/golden/make_config_golden.py",
    }
    for s in case["logit_steps"]:
        row = rows[s]
        top = np.argsort(-row, kind="stable")[:N_TOP]
        idx = np.union1d(top, logit_sample_indices(shape.vocab, s))
        out["logit_samples"].append({"step": s, "idx": [int(i) for i in idx],
                                     "val": [float(row[i]) for i in idx]})
    if sampled:
        cands = []
        for s in range(len(out["ids"])):
            row = rows[s]
            top = np.argsort(-row, kind="stable")[:N_CAND]
            cands.append({"ids": [int(i) for i in top], "logits": [float(row[i]) for i in top]})
        out["candidates"] = cands
    if case.get("experts"):
        ex = res["experts"]  # [forward][layer][k], prompt forwards first
        out["experts"] = ex.tolist()
    return out


def main(argv: list[str]) -> None:
    if not oracle_py.ref_available():
        sys.exit("oracle/_ref is not built (make -C oracle REF=<reference checkout> ref)")
    names = argv or list(CASES)
    model_dir = Path(os.environ.get("MF_MODEL_DIR", "/dev/shm/minfer_b200_cfg"))
    model_dir.mkdir(parents=True, exist_ok=True)
    for name in names:
        g = make(name, model_dir)
        f = HERE / f"config_{name}.json"
        f.write_text(json.dumps(g, separators=(",", ":")) + "\n")
        print(f"{f.name}: {len(g['ids'])} ids, min margin {min(g['margins']):.3g}")


if __name__ == "__main__":
    main(sys.argv[1:])
