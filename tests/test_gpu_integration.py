"""The reference's own host loop on the CUDA runtime (integration/cuda_backend.cpp):
minfer's BaseModel, Config, RunState, Sampler and GGUF reader compiled from
its sources, forward() running through libminfer_host.

* generate: the reference's prompt -> sample -> forward loop with the
  reference's Sampler on this runtime's logits reproduces the reference CPU
  run's greedy ids (golden fixture made by the reference's CPU build; margin
  rule as in the other parity tests);
* bench: the reference's BaseModel::benchmark (pp512 + tg128) runs unchanged
  and reports its statistics.
The binary is built where the reference sources exist and travels with the
working tree.
"""
import json
import subprocess
from pathlib import Path

import numpy as np
import pytest

from conftest import tiny_model

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
APP = ROOT / "integration" / "_build" / "minfer_cuda_app"
GOLDEN = Path(__file__).resolve().parent / "golden"
MARGIN_TOL = 1e-4


def run_app(*args) -> dict:
    assert APP.exists(), "integration/_build/minfer_cuda_app was not built (make -C integration REF=<reference checkout>)"
    r = subprocess.run([str(APP), *map(str, args)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("{")][-1])


@pytest.mark.parametrize("fixture", ["model_tiny-bf16_greedy.json", "model_tiny-f32_greedy.json",
                                     "model_tiny-moe_greedy.json"])
def test_reference_loop_greedy_on_cuda(gpu, tmp_path, fixture):
    g = json.loads((GOLDEN / fixture).read_text())
    pf = tmp_path / "prompt.u32"
    np.array(g["prompt"], np.uint32).tofile(pf)
    out = run_app("generate", tiny_model(g["model"]), "--prompt-file", pf, "--gen", len(g["ids"]))
    ids = out["ids"]
    assert len(ids) == len(g["ids"])
    first = next((i for i, (a, b) in enumerate(zip(ids, g["ids"])) if a != b), None)
    if first is not None:  # free-running: identical up to a near-tie of the reference's logits
        assert g["margins"][first] < MARGIN_TOL, f"id {first} differs, margin {g['margins'][first]}"


def test_reference_benchmark_on_cuda(gpu):
    out = run_app("bench", tiny_model("tiny-bf16"), "--seed", 30, "--max-seq", 1024)
    assert out["num_tokens_gen"] == 128
    assert out["throughput"] > 0 and out["prefill_time"] > 0 and out["bandwidth"] > 0


def test_reference_text_loop_on_cuda(gpu):
    """The reference's BaseModel::generate(std::string&), unchanged, with this
    runtime's tokenizer behind its BaseTokenizer interface and this runtime's
    forward: it prints the chat-template prompt, the token count and the
    generated text that the Python runtime produces for the same prompt
    (token-by-token prefill on both sides, so the logits are the same)."""
    from conftest import text_model
    from minfer_b200.model import Qwen3Model, RunParams
    from minfer_b200.tokenizer import Qwen3Tokenizer

    path = text_model()
    text = "Hello, world! It's 2 + 2 = 4"
    G = 24
    assert APP.exists(), "integration/_build/minfer_cuda_app was not built (make -C integration REF=<reference checkout>)"
    r = subprocess.run([str(APP), "text", path, "--prompt", text, "--gen", str(G), "--max-seq", "256"],
                       capture_output=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    out = r.stdout
    tok = Qwen3Tokenizer.from_gguf(path)
    formatted = tok.apply_chat_template([{"role": "user", "content": text}], [], True)
    prompt = tok.encode(formatted)
    assert b"Formatted message:\n" + formatted.encode() + b"\n" in out
    assert b"Number of tokens: %d\n" % len(prompt) in out
    m = Qwen3Model(path, RunParams(num_iters=G, max_seq_len=256)).set_device("cuda")
    ids, _, _ = m.generate(prompt, G, stop_at_eos=True, token_prefill=True)
    n = len(prompt)
    assert b"Prefill progress: %d/%d\r\n" % (n, n) + tok.decode(ids) + b"\n\n" in out
    summary = json.loads([ln for ln in out.decode(errors="replace").splitlines() if ln.startswith("{")][-1])
    assert summary["num_tokens_gen"] == len(ids)
