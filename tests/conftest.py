import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

from minfer_b200.gguf_synth import Qwen3Shape, ensure_gguf  # noqa: E402

# Small synthetic models shared by the parity tests. d_head is 128 (the
# decode-attention kernel's head size, as in every Qwen3 model).
TINY = {
    "tiny-bf16": Qwen3Shape(2, 256, 4, 2, 128, 512, 1024, "bf16", True, seed=101),
    "tiny-f32": Qwen3Shape(2, 256, 4, 2, 128, 512, 1024, "f32", False, seed=102),
    "tiny-f16": Qwen3Shape(2, 256, 4, 2, 128, 512, 1024, "f16", True, seed=103),
    "tiny-gqa8": Qwen3Shape(2, 256, 16, 2, 128, 384, 1024, "bf16", False, seed=104),
    "tiny-moe": Qwen3Shape(2, 256, 4, 2, 128, 128, 1024, "bf16", False, 16, 4, seed=105),
    # 8 KV heads: tensor-parallel splits up to 8 ranks
    "tiny-tp8": Qwen3Shape(2, 512, 16, 8, 128, 1024, 2048, "bf16", False, seed=106),
}


# a tiny model whose GGUF carries a byte-level BPE vocabulary and the ChatML
# template: text prompts run end to end (tokenizer -> GPU decode -> text)
TEXT_MODEL = Qwen3Shape(2, 256, 4, 2, 128, 512, 1024, "bf16", True, seed=107, byte_vocab=True)


def text_model() -> str:
    return ensure_gguf(model_dir() / "tiny-text.gguf", TEXT_MODEL)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")
    config.addinivalue_line("markers", "slow: long-running parity case")


def model_dir() -> Path:
    d = Path(os.environ.get("MF_MODEL_DIR", "/tmp/minfer_b200_models"))
    d.mkdir(parents=True, exist_ok=True)
    return d


def tiny_model(name: str) -> str:
    return ensure_gguf(model_dir() / f"{name}.gguf", TINY[name])


@pytest.fixture(scope="session")
def models():
    return {name: tiny_model(name) for name in TINY}


@pytest.fixture(scope="session")
def gpu():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    from minfer_b200 import model as mm

    mm.init(1, [0])
    return torch.device("cuda:0")
