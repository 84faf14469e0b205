"""Writes the model-level golden fixtures of tests/golden/ by running the
reference's own CPU token loop (oracle/_ref/minfer_ref_run, built from the
reference sources) on the seeded synthetic GGUF models of tests/conftest.py.

Run from the repository root in the development container:
    python tests/golden/make_golden.py
Each fixture holds the prompt, the sampler settings, the generated ids, the
top-2 margin and top-1 logit of every decode step, and the full logits of the
first decode step.
"""
import json
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE.parent))

from conftest import TINY, tiny_model  # noqa: E402
from minfer_b200.gguf_synth import random_prompt  # noqa: E402
from oracle.oracle_py import ref_available, run_reference  # noqa: E402

CASES = [
    # (model, prompt len, prompt seed, decode steps, sampler settings)
    ("tiny-bf16", 12, 30, 32, dict(temp=0.0, top_k=1, top_p=1.0, seed=0)),
    ("tiny-f32", 12, 31, 32, dict(temp=0.0, top_k=1, top_p=1.0, seed=0)),
    ("tiny-f16", 12, 32, 32, dict(temp=0.0, top_k=1, top_p=1.0, seed=0)),
    ("tiny-gqa8", 12, 33, 32, dict(temp=0.0, top_k=1, top_p=1.0, seed=0)),
    ("tiny-moe", 12, 34, 32, dict(temp=0.0, top_k=1, top_p=1.0, seed=0)),
    ("tiny-bf16", 16, 42, 48, dict(temp=0.7, top_k=20, top_p=0.9, seed=42)),
]


def main():
    if not ref_available():
        sys.exit("oracle/_ref is not built (make -C oracle REF=<reference checkout> ref)")
    for model, P, pseed, G, smp in CASES:
        path = tiny_model(model)
        prompt = random_prompt(P, TINY[model].vocab, pseed)
        with tempfile.TemporaryDirectory() as td:
            res = run_reference(path, f"{td}/r", prompt=prompt, gen=G, max_seq=P + G + 1, dump_logits=[0], **smp)
        mode = "greedy" if smp["temp"] == 0 else "sampled"
        out = {
            "model": model,
            "source": "reference CPU path (oracle/_ref/minfer_ref_run)",
            "prompt": [int(t) for t in prompt],
            "sampler": {"top_k": smp["top_k"], "temp": smp["temp"], "top_p": smp["top_p"], "seed": smp["seed"]},
            "ids": res["ids"],
            "margins": res["margins"],
            "top1": res["top1"],
            "logits_step0": [float(v) for v in res["logits"][0]],
        }
        if "experts" in res:
            out["experts"] = res["experts"].tolist()
        fn = HERE / f"model_{model}_{mode}.json"
        fn.write_text(json.dumps(out, separators=(",", ":")))
        print("wrote", fn.name, "ids", res["ids"][:8], "...")


if __name__ == "__main__":
    main()
