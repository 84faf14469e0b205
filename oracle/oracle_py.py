"""ORACLE — test infrastructure only (imported by tests/, __graft_entry__.smoke
and bench.py's CPU-baseline leg; never by the product).

ctypes access to
  * _build/liboracle.so      the restatement of the reference's CPU algorithm
                             (qwen3_oracle.cpp), and
  * _ref/libminfer_ref_ops.so, _ref/minfer_ref_run
                             the reference's own CPU code compiled from its
                             sources (present when built in the development
                             container; travels with the working tree).
"""
from __future__ import annotations

import ctypes as C
import json
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PORT_LIB = HERE / "_build" / "liboracle.so"
REF_OPS_LIB = HERE / "_ref" / "libminfer_ref_ops.so"
REF_RUN = HERE / "_ref" / "minfer_ref_run"
REF_RUN_NATIVE = HERE / "_ref" / "minfer_ref_run_native"  # -march=native of the build machine
REF_NATIVE_FLAGS = HERE / "_ref" / "native_flags.txt"  # that machine's CPU flags

P, I, U32, SZ, F = C.c_void_p, C.c_int, C.c_uint32, C.c_size_t, C.c_float

_OPS_SIG = {
    "silu": (F, [F]),
    "softmax": (None, [P, P, I]),
    "il_rope": (None, [P, P, I, I, I, F, I]),
    "neox_rope": (None, [P, P, I, I, I, F, I]),
    "attn": (None, [P, P, P, P, P, I, I, I]),
    "rmsnorm": (None, [P, P, P, I, F]),
    "route": (None, [P, P, P, P, P, I, I, I]),
}


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


class _Ops:
    """The reference's op set (include/minfer/ops/kernels.hpp) on numpy arrays."""

    def __init__(self, lib: C.CDLL, prefix: str):
        self.lib = lib
        self.prefix = prefix
        for name, (res, args) in _OPS_SIG.items():
            fn = getattr(lib, prefix + name)
            fn.restype, fn.argtypes = res, args

    def silu(self, x: float) -> float:
        return getattr(self.lib, self.prefix + "silu")(x)

    def softmax(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        getattr(self.lib, self.prefix + "softmax")(_ptr(out), _ptr(x), x.size)
        return out

    def rope(self, x, head, d_head, d_rot, base, pos, neox=True, out=None):
        x = np.ascontiguousarray(x, np.float32)
        out = x.copy() if out is None else out
        fn = getattr(self.lib, self.prefix + ("neox_rope" if neox else "il_rope"))
        fn(_ptr(out), _ptr(x), head, d_head, d_rot, base, pos)
        return out

    def attn(self, q, k, v, seq_len, d_head, kv_dim):
        q, k, v = (np.ascontiguousarray(a, np.float32) for a in (q, k, v))
        scores = np.zeros(seq_len, np.float32)
        out = np.zeros(d_head, np.float32)
        getattr(self.lib, self.prefix + "attn")(_ptr(scores), _ptr(out), _ptr(q), _ptr(k), _ptr(v), seq_len, d_head,
                                                kv_dim)
        return scores, out

    def rmsnorm(self, x, w, eps):
        x, w = np.ascontiguousarray(x, np.float32), np.ascontiguousarray(w, np.float32)
        out = np.empty_like(x)
        getattr(self.lib, self.prefix + "rmsnorm")(_ptr(out), _ptr(x), _ptr(w), x.size, eps)
        return out

    def route(self, x, w_router, n_experts, k):
        x, w_router = np.ascontiguousarray(x, np.float32), np.ascontiguousarray(w_router, np.float32)
        ids = np.zeros(k, np.int32)
        wts = np.zeros(k, np.float32)
        scores = np.zeros(n_experts, np.float32)
        getattr(self.lib, self.prefix + "route")(_ptr(x), _ptr(ids), _ptr(wts), _ptr(scores), _ptr(w_router),
                                                 x.size, n_experts, k)
        return ids, wts, scores


class PortOps(_Ops):
    def __init__(self):
        lib = C.CDLL(str(PORT_LIB))
        super().__init__(lib, "orc_")
        lib.orc_matmul.restype = None
        lib.orc_matmul.argtypes = [P, P, P, I, SZ, I, I]
        lib.orc_embed.restype = None
        lib.orc_embed.argtypes = [P, P, I, U32, SZ]

    def matmul(self, x, w, dtype: int, offset: int, d_out: int, d_in: int) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(d_out, np.float32)
        self.lib.orc_matmul(_ptr(out), _ptr(x), _ptr(np.ascontiguousarray(w)), dtype, offset, d_out, d_in)
        return out

    def embed(self, w, dtype: int, token: int, d: int) -> np.ndarray:
        out = np.zeros(d, np.float32)
        self.lib.orc_embed(_ptr(out), _ptr(np.ascontiguousarray(w)), dtype, token, d)
        return out


class RefOps(_Ops):
    """The reference's own ops (compiled from its sources)."""

    def __init__(self):
        lib = C.CDLL(str(REF_OPS_LIB))
        super().__init__(lib, "ref_")
        for n, wt in (("f32", P), ("f16", P), ("bf16", P)):
            fn = getattr(lib, f"ref_matmul_{n}")
            fn.restype, fn.argtypes = None, [P, P, wt, SZ, I, I]
            fe = getattr(lib, f"ref_embed_{n}")
            fe.restype, fe.argtypes = None, [P, P, U32, SZ]

    def matmul(self, x, w, dtype: int, offset: int, d_out: int, d_in: int) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(d_out, np.float32)
        name = {0: "f32", 1: "f16", 2: "bf16"}[dtype]
        getattr(self.lib, f"ref_matmul_{name}")(_ptr(out), _ptr(x), _ptr(np.ascontiguousarray(w)), offset, d_out,
                                                d_in)
        return out

    def embed(self, w, dtype: int, token: int, d: int) -> np.ndarray:
        out = np.zeros(d, np.float32)
        name = {0: "f32", 1: "f16", 2: "bf16"}[dtype]
        getattr(self.lib, f"ref_embed_{name}")(_ptr(out), _ptr(np.ascontiguousarray(w)), token, d)
        return out


def uniform_draws(seed: int, n: int) -> np.ndarray:
    """The first n random numbers the reference's Sampler draws with this seed
    (one per sampled token)."""
    lib = C.CDLL(str(PORT_LIB))
    lib.orc_uniform_draws.restype = None
    lib.orc_uniform_draws.argtypes = [I, SZ, P]
    out = np.zeros(n, np.float32)
    lib.orc_uniform_draws(seed, n, _ptr(out))
    return out


def port_available() -> bool:
    return PORT_LIB.exists()


def ref_available() -> bool:
    return REF_OPS_LIB.exists() and REF_RUN.exists()


class PortModel:
    """The oracle token loop (restatement) over a GGUF file."""

    def __init__(self, path: str, max_seq: int, top_k: int = 1, temp: float = 0.0, top_p: float = 1.0,
                 min_p: float = 0.0, pres: float = 0.0, seed: int = 0, kv_bf16: bool = False):
        """kv_bf16 emulates the CUDA runtime's opt-in bf16 KV cache (appended
        rows rounded to bf16, nearest even); the reference has no such option."""
        lib = C.CDLL(str(PORT_LIB))
        lib.orc_model_open.restype = P
        lib.orc_model_open.argtypes = [C.c_char_p, SZ, SZ, F, F, F, F, I]
        lib.orc_model_close.argtypes = [P]
        lib.orc_model_vocab.restype = I
        lib.orc_model_vocab.argtypes = [P]
        lib.orc_model_forward.argtypes = [P, U32, I, I]
        lib.orc_model_logits.restype = C.POINTER(C.c_float)
        lib.orc_model_logits.argtypes = [P]
        lib.orc_model_kv.argtypes = [P, I, I, P, P]
        lib.orc_generate.restype = SZ
        lib.orc_generate.argtypes = [P, P, SZ, SZ, P, P]
        lib.orc_model_record_experts.argtypes = [P, I]
        lib.orc_model_recorded.restype = SZ
        lib.orc_model_recorded.argtypes = [P, P, P]
        lib.orc_sample.restype = U32
        lib.orc_sample.argtypes = [P, P]
        lib.orc_sampler_add.argtypes = [P, U32]
        self.lib = lib
        self.h = lib.orc_model_open(str(path).encode(), max_seq, top_k, temp, top_p, min_p, pres, seed)
        if not self.h:
            raise RuntimeError(f"oracle could not open {path}")
        self.vocab = lib.orc_model_vocab(self.h)
        if kv_bf16:
            lib.orc_model_set_kv_bf16.argtypes = [P, I]
            lib.orc_model_set_kv_bf16(self.h, 1)

    def close(self):
        if self.h:
            self.lib.orc_model_close(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def forward(self, token: int, pos: int, logits: bool = True):
        self.lib.orc_model_forward(self.h, token, pos, int(logits))

    def logits(self) -> np.ndarray:
        return np.ctypeslib.as_array(self.lib.orc_model_logits(self.h), shape=(self.vocab,)).copy()

    def kv(self, layer: int, n_pos: int, kv_dim: int):
        k = np.zeros(n_pos * kv_dim, np.float32)
        v = np.zeros(n_pos * kv_dim, np.float32)
        self.lib.orc_model_kv(self.h, layer, n_pos, _ptr(k), _ptr(v))
        return k, v

    def record_experts(self, on: bool = True):
        self.lib.orc_model_record_experts(self.h, int(on))

    def recorded_experts(self, k: int):
        n = self.lib.orc_model_recorded(self.h, None, None)
        ids = np.zeros(n, np.int32)
        w = np.zeros(n, np.float32)
        self.lib.orc_model_recorded(self.h, _ptr(ids), _ptr(w))
        return ids.reshape(-1, k), w.reshape(-1, k)

    def sample(self, logits: np.ndarray) -> int:
        logits = np.ascontiguousarray(logits, np.float32)
        return int(self.lib.orc_sample(self.h, _ptr(logits)))

    def add_token(self, tok: int):
        self.lib.orc_sampler_add(self.h, tok)

    def generate(self, prompt, n_gen: int):
        prompt = np.ascontiguousarray(prompt, np.uint32)
        out = np.zeros(n_gen, np.uint32)
        mg = np.zeros(n_gen, np.float32)
        n = self.lib.orc_generate(self.h, _ptr(prompt), prompt.size, n_gen, _ptr(out), _ptr(mg))
        return out[:n], mg[:n]


def ref_binary() -> tuple[Path, str]:
    """The reference token-loop build to run here and its arch flags: the
    -march=native build when this CPU has every flag of the machine it was
    built on (so every instruction it may use exists here), else x86-64-v3."""
    try:
        want = set(REF_NATIVE_FLAGS.read_text().split())
        have = set()
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    have = set(line.split(":", 1)[1].split())
                    break
        if REF_RUN_NATIVE.exists() and want and want <= have:
            return REF_RUN_NATIVE, "-march=native (this CPU's flags include the build machine's)"
    except OSError:
        pass
    return REF_RUN, "-march=x86-64-v3"


def run_reference(model: str, out_prefix: str, *, prompt=None, random_prompt: int = 0, prompt_seed: int = 0,
                  gen: int = 8, max_seq: int = 0, temp: float = 0.0, top_k: int = 1, top_p: float = 1.0,
                  min_p: float = 0.0, pres: float = 0.0, seed: int = 0, dump_logits=(), threads: int | None = None,
                  bench_context: int = -1, bench_steps: int = 0, bench_warmup: int = 0, llama_bench: bool = False,
                  timeout: float = 3600):
    """Run the reference's own CPU token loop (minfer_ref_run) and load its dump."""
    binary, _ = ref_binary()
    args = [str(binary), str(model), "--out", out_prefix, "--gen", str(gen), "--temp", str(temp), "--top-k",
            str(top_k), "--top-p", str(top_p), "--min-p", str(min_p), "--pres", str(pres), "--seed", str(seed)]
    if prompt is not None:
        pf = out_prefix + ".prompt.u32"
        np.ascontiguousarray(prompt, np.uint32).tofile(pf)
        args += ["--prompt-file", pf]
    if random_prompt:
        args += ["--random-prompt", str(random_prompt), "--prompt-seed", str(prompt_seed)]
    if max_seq:
        args += ["--max-seq", str(max_seq)]
    if dump_logits:
        args += ["--dump-logits", ",".join(str(s) for s in dump_logits)]
    if bench_context >= 0:
        args += ["--bench-context", str(bench_context), "--bench-steps", str(bench_steps), "--bench-warmup",
                 str(bench_warmup), "--prompt-seed", str(prompt_seed)]
    if llama_bench:
        args += ["--llama-bench"]
    env = dict(os.environ)
    if threads:
        env["OMP_NUM_THREADS"] = str(threads)
    subprocess.run(args, check=True, env=env, timeout=timeout, stdout=subprocess.DEVNULL)
    with open(out_prefix + ".json") as f:
        res = json.load(f)
    if res.get("mode") == "generate":
        V = res["vocab"]
        lg = np.fromfile(out_prefix + ".logits.f32", dtype=np.float32)
        res["logits"] = lg.reshape(-1, V) if lg.size else np.zeros((0, V), np.float32)
        ex = np.fromfile(out_prefix + ".experts.bin", dtype=np.int32)
        k = res.get("k", 0)
        if ex.size and k:
            half = ex.size // 2
            res["experts"] = ex[:half].reshape(-1, res["n_layers"], k)
            res["expert_w"] = ex[half:].view(np.float32).reshape(-1, res["n_layers"], k)
    return res
