"""Python face of the CUDA host runtime (include/minfer_model.h), shaped like
the reference's BaseModel / Qwen3Model (include/minfer/base/model.hpp:17-41,
include/minfer/models/qwen3/model.hpp): construct from a GGUF path and
RunParams, `set_device("cuda")`, then `forward`, `generate`, `benchmark`.
Token ids stand in for text (the tokenizer is not on this path).
"""
from __future__ import annotations

import ctypes as C
import dataclasses

import numpy as np

from ._lib import (MF_BF16, MF_COMM_HANDLE_BYTES, MF_E_UNSUPPORTED, MF_GEN_MARGINS, MF_GEN_STOP_AT_EOS,
                   MF_GEN_TOKEN_PREFILL, MinferError, check, cuda_lib, host_lib, mf_gen_stats, mf_model_info, mf_run_params)


@dataclasses.dataclass
class RunParams:
    """include/minfer/base/config.hpp:37-51."""

    num_iters: int = 0
    max_seq_len: int = 4096
    top_k: int = 1
    temp: float = 0.0
    top_p: float = 1.0
    min_p: float = 0.0
    penalty_pres: float = 0.0
    seed: int = 0

    def to_c(self) -> mf_run_params:
        return mf_run_params(self.num_iters, self.max_seq_len, self.top_k, self.temp, self.top_p, self.min_p,
                             self.penalty_pres, self.seed)


@dataclasses.dataclass
class GenStats:
    """include/minfer/base/stats.hpp:3-15."""

    num_tokens_gen: int
    ttft: float
    throughput: float
    prefill_time: float
    bandwidth: float
    decode_seconds: float
    bytes_read: float


_initialised: set = set()


def init(n_ranks: int = 1, devices: list[int] | None = None) -> None:
    """MetalManager::init equivalent: pick devices, create per-rank streams."""
    key = (n_ranks, tuple(devices) if devices else None)
    if key in _initialised:
        return
    arr = (C.c_int * n_ranks)(*(devices or range(n_ranks)))
    check(cuda_lib().mf_init(n_ranks, arr))
    _initialised.add(key)


@dataclasses.dataclass
class TextResult:
    formatted: str          # the chat-template prompt
    prompt_ids: list[int]
    ids: list[int]          # generated ids (EOS included when reached)
    text: bytes             # the generated ids decoded
    stats: "GenStats"


class Qwen3Model:
    """`tp_rank`/`tp_size` > 1 loads this process's tensor-parallel shard
    (dense models); after `set_device("cuda")` connect the ranks with
    `minfer_b200.tp.connect` (or comm_handle / comm_connect directly).
    `kv_dtype` "bf16" opts into a bf16 KV cache (the reference keeps fp32):
    half the cache bytes, every appended row rounded to nearest even."""

    def __init__(self, model_file: str, run_params: RunParams, rank: int = 0, device: int | None = None,
                 tp_rank: int = 0, tp_size: int = 1, kv_dtype: str = "f32"):
        if not _initialised:
            init(1, [device if device is not None else 0])
        self._lib = host_lib()
        self._h = C.c_void_p()
        self.model_file = str(model_file)
        self._tokenizer = None
        self.run_params = run_params
        self._rp = run_params.to_c()
        check(self._lib.mf_model_load_tp(str(model_file).encode(), C.byref(self._rp), rank, tp_rank, tp_size,
                                         C.byref(self._h)))
        if kv_dtype not in ("f32", "bf16"):
            raise ValueError(f"kv_dtype {kv_dtype!r}: f32 or bf16")
        if kv_dtype != "f32":
            check(self._lib.mf_model_set_kv_dtype(self._h, MF_BF16))
        self.kv_dtype = kv_dtype
        self.device = "cpu"
        self._refresh_info()

    def _refresh_info(self):
        info = mf_model_info()
        check(self._lib.mf_model_info_get(self._h, C.byref(info)))
        self.info = info
        self.vocab_size = info.vocab_size

    def set_device(self, device: str) -> "Qwen3Model":
        if device != "cuda":
            raise ValueError("this runtime runs the model on CUDA only")
        check(self._lib.mf_model_to_cuda(self._h))
        self.device = "cuda"
        self._refresh_info()
        return self

    def close(self):
        if self._h:
            self._lib.mf_model_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- tensor parallelism
    def comm_handle(self) -> bytes:
        buf = (C.c_char * MF_COMM_HANDLE_BYTES)()
        check(self._lib.mf_model_comm_handle(self._h, buf, MF_COMM_HANDLE_BYTES))
        return bytes(buf)

    def comm_connect(self, handles: list[bytes]) -> None:
        blob = b"".join(handles)
        if len(handles) != self.info.tp_size or len(blob) != len(handles) * MF_COMM_HANDLE_BYTES:
            raise ValueError("need one handle of MF_COMM_HANDLE_BYTES per tensor-parallel rank")
        buf = C.create_string_buffer(blob, len(blob))
        check(self._lib.mf_model_comm_connect(self._h, buf, len(blob)))

    def comm_status(self) -> int:
        v = C.c_int()
        check(self._lib.mf_model_comm_status(self._h, C.byref(v)))
        return v.value

    # -- BaseModel::forward
    def forward(self, token: int, pos: int, compute_logits: bool = True, host_logits: bool = True):
        check(self._lib.mf_model_forward(self._h, int(token), int(pos), int(compute_logits), int(host_logits)))

    def logits(self) -> np.ndarray:
        out = np.empty(self.vocab_size, dtype=np.float32)
        check(self._lib.mf_model_logits(self._h, out.ctypes.data, self.vocab_size))
        return out

    def argmax(self) -> int:
        v = C.c_uint32()
        check(self._lib.mf_model_argmax(self._h, C.byref(v)))
        return v.value

    # -- batched prefill (tensor cores); False when the model is not eligible
    def prefill(self, tokens, pos0: int = 0, compute_logits: bool = True, host_logits: bool = True) -> bool:
        tokens = np.ascontiguousarray(tokens, dtype=np.uint32)
        rc = self._lib.mf_model_prefill(self._h, tokens.ctypes.data, tokens.size, int(pos0), int(compute_logits),
                                        int(host_logits))
        if rc == MF_E_UNSUPPORTED:
            return False
        check(rc)
        return True

    # -- BaseModel::generate (ids in, ids out)
    def generate(self, prompt, n_gen: int, stop_at_eos: bool = False, forced=None, margins: bool = False,
                 token_prefill: bool = False, logits_at=None):
        """Ids (and margins, stats). With `logits_at` (a list of step numbers)
        a fourth result holds the logits each of those steps drew from."""
        prompt = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.zeros(n_gen, dtype=np.uint32)
        mg = np.zeros(n_gen, dtype=np.float32)
        n_out = C.c_size_t()
        st = mf_gen_stats()
        flags = ((MF_GEN_STOP_AT_EOS if stop_at_eos else 0) | (MF_GEN_MARGINS if margins else 0) |
                 (MF_GEN_TOKEN_PREFILL if token_prefill else 0))
        forced_arr = None if forced is None else np.ascontiguousarray(forced, dtype=np.uint32)
        steps = np.ascontiguousarray(logits_at if logits_at is not None else [], dtype=np.uintp)
        lg = np.zeros((steps.size, self.vocab_size), dtype=np.float32)
        check(self._lib.mf_model_generate_logits(self._h, prompt.ctypes.data, prompt.size, n_gen, flags,
                                                 None if forced_arr is None else forced_arr.ctypes.data,
                                                 out.ctypes.data, C.byref(n_out), mg.ctypes.data, C.byref(st),
                                                 steps.ctypes.data if steps.size else None, steps.size,
                                                 lg.ctypes.data if steps.size else None))
        n = n_out.value
        stats = GenStats(st.num_tokens_gen, st.ttft, st.throughput, st.prefill_time, st.bandwidth,
                         st.decode_seconds, st.bytes_read)
        if logits_at is not None:
            return out[:n], (mg[:n] if margins else None), stats, lg
        return out[:n], (mg[:n] if margins else None), stats

    # -- BaseModel::generate(std::string&) (src/base/model.cpp:99-186)
    def generate_text(self, text: str, n_gen: int | None = None) -> "TextResult":
        """One user message through the model file's chat template
        (add_generation_prompt), encoded by its tokenizer, then the token loop
        until EOS or min(num_iters, max_seq_len - prompt length) tokens, as
        the reference's generate does; the output keeps the EOS token. The
        tokenizer runs on the host (minfer_b200.tokenizer)."""
        from .tokenizer import Qwen3Tokenizer

        if getattr(self, "_tokenizer", None) is None:
            self._tokenizer = Qwen3Tokenizer.from_gguf(self.model_file)
        tok = self._tokenizer
        formatted = tok.apply_chat_template([{"role": "user", "content": text}], [], True)
        prompt = tok.encode(formatted)
        max_seq = self.run_params.max_seq_len
        if len(prompt) > max_seq:
            raise ValueError(f"{len(prompt)} prompt tokens exceed max_seq_len {max_seq}")
        n = min(self.run_params.num_iters, max_seq - len(prompt)) if n_gen is None else n_gen
        ids, _, stats = self.generate(prompt, n, stop_at_eos=True)
        ids = [int(i) for i in ids]
        return TextResult(formatted, prompt, ids, tok.decode(ids), stats)

    def benchmark(self, token_prefill: bool = False) -> GenStats:
        """BaseModel::benchmark: pp512 then tg128 with random ids (seed from RunParams)."""
        st = mf_gen_stats()
        check(self._lib.mf_model_benchmark(self._h, MF_GEN_TOKEN_PREFILL if token_prefill else 0, C.byref(st)))
        return GenStats(st.num_tokens_gen, st.ttft, st.throughput, st.prefill_time, st.bandwidth,
                        st.decode_seconds, st.bytes_read)

    def decode_chained(self, token: int, start_pos: int, n: int) -> int:
        last = C.c_uint32()
        check(self._lib.mf_model_decode_chained(self._h, int(token), int(start_pos), int(n), C.byref(last)))
        return last.value

    def reset_sampler(self):
        check(self._lib.mf_model_reset_sampler(self._h))

    # -- test access
    def experts(self, layer: int):
        k = self.info.n_active_experts
        ids = np.zeros(k, dtype=np.int32)
        w = np.zeros(k, dtype=np.float32)
        check(self._lib.mf_model_experts(self._h, layer, ids.ctypes.data, w.ctypes.data))
        return ids, w

    def prefill_experts(self, layer: int, n_tokens: int):
        """Expert ids / weights ([n_tokens][k]) the last batched prefill chose at `layer`."""
        k = self.info.n_active_experts
        ids = np.zeros((n_tokens, k), dtype=np.int32)
        w = np.zeros((n_tokens, k), dtype=np.float32)
        check(self._lib.mf_model_prefill_experts(self._h, layer, ids.ctypes.data, w.ctypes.data, n_tokens))
        return ids, w

    def kv(self, layer: int, n_pos: int):
        # tensor parallelism splits the KV heads; expert parallelism (MoE) keeps them all
        kvh = self.info.n_kv_heads if self.info.expert_parallel else self.info.n_kv_heads // self.info.tp_size
        n = n_pos * kvh * self.info.d_head
        k = np.zeros(n, dtype=np.float32)
        v = np.zeros(n, dtype=np.float32)
        check(self._lib.mf_model_kv(self._h, layer, k.ctypes.data, v.ctypes.data, n_pos))
        return k, v

    def x(self) -> np.ndarray:
        out = np.zeros(self.info.d_model, dtype=np.float32)
        check(self._lib.mf_model_x(self._h, out.ctypes.data))
        return out


def random_prompt(n: int, vocab: int, seed: int) -> np.ndarray:
    """Prompt ids as BaseModel::benchmark draws them (src/base/model.cpp:189-193)."""
    out = np.zeros(n, dtype=np.uint32)
    check(host_lib().mf_random_prompt(seed, vocab, n, out.ctypes.data))
    return out
