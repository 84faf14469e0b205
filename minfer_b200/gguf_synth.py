"""Seeded synthetic Qwen3 GGUF v3 files.

The reference only loads models from GGUF v3 files (src/parsing/gguf.cpp:145-242,
src/base/config.cpp:171-337), so every parity case and benchmark workload is a
GGUF written here: random N(0, std) weights from numpy's PCG64 with a fixed
seed, norm weights 1.0, a synthetic byte-level BPE vocabulary, and exactly the
metadata keys `Config::Config` requires (src/base/config.cpp:281-325).

Layout rules follow the GGUF spec restated in include/minfer/parsing/gguf.hpp:
little-endian, dims stored innermost first (a logical [out, in] matrix is
written as ne = (in, out)), tensor data aligned to `general.alignment` (32).
"""
from __future__ import annotations

import dataclasses
import os
import struct
from typing import BinaryIO, Iterable

import numpy as np

# value types (include/minfer/parsing/gguf.hpp ValueType)
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STR, _ARR, _U64, _I64, _F64 = range(13)
# tensor types (include/minfer/parsing/gguf.hpp TensorType)
GGML_F32, GGML_F16, GGML_BF16 = 0, 1, 30
_DTYPE_CODE = {"f32": GGML_F32, "f16": GGML_F16, "bf16": GGML_BF16}
_DTYPE_SIZE = {"f32": 4, "f16": 2, "bf16": 2}
ALIGN = 32
MAGIC = 0x46554747


@dataclasses.dataclass(frozen=True)
class Qwen3Shape:
    """Hyper-parameters of a Qwen3-shaped model (dense or MoE)."""

    n_layers: int
    d_model: int
    n_heads: int
    n_kv_heads: int
    d_head: int
    d_ff: int
    vocab: int
    dtype: str = "bf16"
    tied: bool = True
    n_experts: int = 0
    n_active: int = 0
    eps: float = 1e-6
    rope_base: float = 1e6
    context_length: int = 40960
    seed: int = 0
    std: float = 0.02
    # layers of the model whose random streams this file follows (0: n_layers).
    # A file with n_layers < rng_layers is the depth-reduced prefix of that
    # model: the same embedding, layers 0..n_layers-1 and lm_head weights.
    rng_layers: int = 0
    # vocabulary: False = printable-ASCII placeholder strings (ids-only
    # workloads); True = a byte-level BPE vocabulary (all 256 bytes, merges
    # whose results are vocabulary entries, and the Qwen3 chat specials), so
    # the file's tokenizer encodes any text
    byte_vocab: bool = False

    def with_(self, **kw) -> "Qwen3Shape":
        return dataclasses.replace(self, **kw)

    def prefix(self, n_layers: int) -> "Qwen3Shape":
        """The first n_layers decoder layers of this model, with its embedding,
        final norm and lm_head (the same weights, drawn from the same streams)."""
        if not 1 <= n_layers <= self.n_layers:
            raise ValueError("prefix depth outside [1, n_layers]")
        return dataclasses.replace(self, n_layers=n_layers, rng_layers=self.rng_layers or self.n_layers)

    @property
    def moe(self) -> bool:
        return self.n_experts > 0

    def weight_bytes(self) -> int:
        s = _DTYPE_SIZE[self.dtype]
        d, q, kv, f = self.d_model, self.n_heads * self.d_head, self.n_kv_heads * self.d_head, self.d_ff
        per = (q * d + 2 * kv * d + d * q) * s
        per += (3 * f * d * max(self.n_experts, 1)) * s
        per += (self.n_experts * d * 4) if self.moe else 0
        per += (2 * d + 2 * self.d_head) * 4
        tot = per * self.n_layers + self.vocab * d * s * (1 if self.tied else 2) + d * 4
        return tot


# The five model shapes of the workloads (Qwen3-0.6B/1.7B/8B/30B-A3B/32B).
CONFIGS = {
    "qwen3-0.6b-f32": Qwen3Shape(28, 1024, 16, 8, 128, 3072, 151936, "f32", True, seed=42),
    "qwen3-1.7b-bf16": Qwen3Shape(28, 2048, 16, 8, 128, 6144, 151936, "bf16", True, seed=42),
    "qwen3-8b-bf16": Qwen3Shape(36, 4096, 32, 8, 128, 12288, 151936, "bf16", False, seed=7),
    "qwen3-30b-a3b-bf16": Qwen3Shape(48, 2048, 32, 4, 128, 768, 151936, "bf16", False, 128, 8, seed=11),
    "qwen3-32b-bf16": Qwen3Shape(64, 5120, 64, 8, 128, 25600, 151936, "bf16", False, seed=3),
}

# Qwen3 special-token ids (vocabulary of 151936 entries)
QWEN3_ENDOFTEXT = 151643
QWEN3_IM_START = 151644
QWEN3_IM_END = 151645
N_QWEN3_SPECIAL = 26  # ids 151643 .. 151668

CHAT_TEMPLATE = (
    "{%- for message in messages %}{{- '<|im_start|>' + message.role + '\\n' + message.content + "
    "'<|im_end|>' + '\\n' }}{%- endfor %}{%- if add_generation_prompt %}{{- '<|im_start|>assistant\\n' }}{%- endif %}"
)


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 bit patterns (uint16)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    r = u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))
    return (r >> np.uint32(16)).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def cast_weights(a: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "f32":
        return np.ascontiguousarray(a, dtype=np.float32)
    if dtype == "f16":
        return np.ascontiguousarray(a, dtype=np.float32).astype(np.float16)
    if dtype == "bf16":
        return f32_to_bf16_bits(a)
    raise ValueError(dtype)


def synth_vocab(n_vocab: int, seed: int, byte_vocab: bool = False) -> tuple[list[bytes], list[int], list[bytes], int, int]:
    """Byte tokens + seeded random merges + special tokens.

    Returns (tokens, token_types, merges, eos_id, pad_id). Token strings are
    printable ASCII so every metadata string is valid UTF-8 (byte_vocab:
    raw bytes, see synth_byte_vocab).
    """
    if byte_vocab:
        return synth_byte_vocab(n_vocab, seed)
    rng = np.random.Generator(np.random.PCG64(seed ^ 0x5EED))
    toks: list[bytes] = []
    for b in range(256):
        toks.append(bytes([b]) if 0x21 <= b <= 0x7E else b"<0x%02X>" % b)
    if n_vocab >= QWEN3_ENDOFTEXT + N_QWEN3_SPECIAL:
        n_special = N_QWEN3_SPECIAL
        first_special = QWEN3_ENDOFTEXT
        eos, pad = QWEN3_IM_END, QWEN3_ENDOFTEXT
    else:
        n_special = 2
        first_special = n_vocab - 2
        eos, pad = n_vocab - 1, n_vocab - 2
    merges: list[bytes] = []
    n_merge = max(first_special - 256, 0)
    a = rng.integers(0, 256, size=n_merge)
    b = rng.integers(0, 256, size=n_merge)
    for i in range(n_merge):
        left, right = toks[int(a[i])][:6], toks[int(b[i])][:6]
        merges.append(left + b" " + right)
        toks.append(left + right + b"%d" % i)
    types = [1] * len(toks)
    for i in range(n_special):
        toks.append(b"<|special_%d|>" % i)
        types.append(3)
    while len(toks) < n_vocab:  # padding ids (Qwen3 pads its vocabulary)
        toks.append(b"<|pad_%d|>" % len(toks))
        types.append(5)
    return toks[:n_vocab], types[:n_vocab], merges, eos, pad


def synth_byte_vocab(n_vocab: int, seed: int) -> tuple[list[bytes], list[int], list[bytes], int, int]:
    """A byte-level BPE vocabulary in the byte form the reference reads: the
    256 single bytes, seeded merges of two existing entries (mostly letters,
    digits and a leading space) whose results are new entries, then the
    specials <|endoftext|> (pad), <|im_start|>, <|im_end|> (eos) as control
    tokens and unused padding ids."""
    rng = np.random.Generator(np.random.PCG64(seed ^ 0xB17E))
    toks = [bytes([b]) for b in range(256)]
    seen = set(toks)
    alpha = [bytes([c]) for c in b"etaoinshrdlucmfwypvbgkqjxz ETAOINSHRD0123456789.,"]
    specials = [b"<|endoftext|>", b"<|im_start|>", b"<|im_end|>"]
    n_normal = n_vocab - len(specials) - max(2, n_vocab // 64)
    merges: list[bytes] = []
    while len(toks) < n_normal:
        grown = len(toks) > 256
        a = toks[int(rng.integers(256, len(toks)))] if grown and rng.random() >= 0.5 else alpha[int(rng.integers(len(alpha)))]
        b = toks[int(rng.integers(256, len(toks)))] if grown and rng.random() >= 0.7 else alpha[int(rng.integers(len(alpha)))]
        m = a + b
        if m in seen or len(m) > 8:
            continue
        seen.add(m)
        toks.append(m)
        merges.append(a + b" " + b)
    types = [1] * len(toks)
    for sp in specials:
        toks.append(sp)
        types.append(3)
    while len(toks) < n_vocab:
        toks.append(b"<|unused_%d|>" % len(toks))
        types.append(5)
    return toks, types, merges, toks.index(b"<|im_end|>"), toks.index(b"<|endoftext|>")


class _Writer:
    def __init__(self, f: BinaryIO):
        self.f = f

    def u32(self, v):
        self.f.write(struct.pack("<I", v))

    def u64(self, v):
        self.f.write(struct.pack("<Q", v))

    def s(self, v: bytes | str):
        if isinstance(v, str):
            v = v.encode()
        self.u64(len(v))
        self.f.write(v)

    def kv(self, key: str, vtype: int, value):
        self.s(key)
        self.u32(vtype)
        self.val(vtype, value)

    def val(self, vtype: int, value):
        fmt = {_U8: "<B", _I8: "<b", _U16: "<H", _I16: "<h", _U32: "<I", _I32: "<i", _F32: "<f",
               _U64: "<Q", _I64: "<q", _F64: "<d"}
        if vtype in fmt:
            self.f.write(struct.pack(fmt[vtype], value))
        elif vtype == _BOOL:
            self.f.write(struct.pack("<B", 1 if value else 0))
        elif vtype == _STR:
            self.s(value)
        else:
            raise ValueError(vtype)

    def arr(self, key: str, etype: int, values: list):
        self.s(key)
        self.u32(_ARR)
        self.u32(etype)
        self.u64(len(values))
        if etype == _STR:
            buf = bytearray()
            for v in values:
                if isinstance(v, str):
                    v = v.encode()
                buf += struct.pack("<Q", len(v))
                buf += v
            self.f.write(bytes(buf))
        elif etype == _I32:
            self.f.write(np.asarray(values, dtype="<i4").tobytes())
        elif etype == _U32:
            self.f.write(np.asarray(values, dtype="<u4").tobytes())
        else:
            for v in values:
                self.val(etype, v)


def tensor_plan(cfg: Qwen3Shape) -> list[tuple[str, tuple[int, ...], str]]:
    """(name, logical shape (outermost first), dtype) in file and RNG order."""
    d, q, kv, f, D = cfg.d_model, cfg.n_heads * cfg.d_head, cfg.n_kv_heads * cfg.d_head, cfg.d_ff, cfg.d_head
    w = cfg.dtype
    plan = [("token_embd.weight", (cfg.vocab, d), w)]
    for i in range(cfg.n_layers):
        p = f"blk.{i}."
        plan += [
            (p + "attn_norm.weight", (d,), "f32"),
            (p + "attn_q.weight", (q, d), w),
            (p + "attn_k.weight", (kv, d), w),
            (p + "attn_v.weight", (kv, d), w),
            (p + "attn_output.weight", (d, q), w),
            (p + "attn_q_norm.weight", (D,), "f32"),
            (p + "attn_k_norm.weight", (D,), "f32"),
            (p + "ffn_norm.weight", (d,), "f32"),
        ]
        if cfg.moe:
            E = cfg.n_experts
            plan += [
                (p + "ffn_gate_inp.weight", (E, d), "f32"),
                (p + "ffn_gate_exps.weight", (E, f, d), w),
                (p + "ffn_up_exps.weight", (E, f, d), w),
                (p + "ffn_down_exps.weight", (E, d, f), w),
            ]
        else:
            plan += [
                (p + "ffn_gate.weight", (f, d), w),
                (p + "ffn_up.weight", (f, d), w),
                (p + "ffn_down.weight", (d, f), w),
            ]
    plan.append(("output_norm.weight", (d,), "f32"))
    if not cfg.tied:
        plan.append(("output.weight", (cfg.vocab, d), w))
    return plan


def rng_index(cfg: Qwen3Shape, plan_index: int) -> int:
    """Random-stream index of the tensor at plan_index: its index in the plan of
    the model with rng_layers layers (tensors after the decoder layers shift)."""
    full = cfg.rng_layers or cfg.n_layers
    if full == cfg.n_layers:
        return plan_index
    per = (len(tensor_plan(cfg)) - 2 - (0 if cfg.tied else 1)) // cfg.n_layers
    first_after = 1 + cfg.n_layers * per
    return plan_index if plan_index < first_after else plan_index + (full - cfg.n_layers) * per


def _is_norm(name: str) -> bool:
    return name.endswith("_norm.weight")


def _align(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


def _fill_chunk(fd: int, file_off: int, seed: int, t_idx: int, c_idx: int, n: int, dt: str, std: float) -> None:
    # every chunk has its own stream: SeedSequence([seed, tensor, chunk]) -> PCG64
    rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, t_idx, c_idx])))
    a = rng.standard_normal(n, dtype=np.float32)
    a *= np.float32(std)
    buf = cast_weights(a, dt).tobytes()
    view = memoryview(buf)
    done = 0
    while done < len(buf):
        done += os.pwrite(fd, view[done:], file_off + done)


def _layout(cfg: Qwen3Shape) -> tuple[bytes, list[tuple], list[int], int, int]:
    """(header bytes up to the aligned data start, tensor plan, tensor offsets
    relative to the data start, data start, data bytes) of the file for cfg."""
    import io

    plan = tensor_plan(cfg)
    toks, types, merges, eos, pad = synth_vocab(cfg.vocab, cfg.seed, cfg.byte_vocab)
    fh = io.BytesIO()
    w = _Writer(fh)
    kvs: list[tuple] = []
    arch = "qwen3"
    kvs.append(("general.architecture", _STR, arch))
    kvs.append(("general.name", _STR, "synthetic-qwen3"))
    kvs.append(("general.alignment", _U32, ALIGN))
    kvs.append((f"{arch}.context_length", _U32, cfg.context_length))
    kvs.append((f"{arch}.embedding_length", _U32, cfg.d_model))
    kvs.append((f"{arch}.block_count", _U32, cfg.n_layers))
    kvs.append((f"{arch}.attention.head_count", _U32, cfg.n_heads))
    kvs.append((f"{arch}.attention.head_count_kv", _U32, cfg.n_kv_heads))
    kvs.append((f"{arch}.attention.key_length", _U32, cfg.d_head))
    kvs.append((f"{arch}.attention.value_length", _U32, cfg.d_head))
    if cfg.moe:
        kvs.append((f"{arch}.expert_feed_forward_length", _U32, cfg.d_ff))
        kvs.append((f"{arch}.feed_forward_length", _U32, cfg.d_ff))
        kvs.append((f"{arch}.expert_count", _U32, cfg.n_experts))
        kvs.append((f"{arch}.expert_used_count", _U32, cfg.n_active))
    else:
        kvs.append((f"{arch}.feed_forward_length", _U32, cfg.d_ff))
    kvs.append((f"{arch}.attention.layer_norm_rms_epsilon", _F32, cfg.eps))
    kvs.append((f"{arch}.rope.freq_base", _F32, cfg.rope_base))
    kvs.append(("tokenizer.ggml.model", _STR, "gpt2"))
    kvs.append(("tokenizer.ggml.pre", _STR, "qwen2"))
    kvs.append(("tokenizer.ggml.eos_token_id", _U32, eos))
    kvs.append(("tokenizer.ggml.padding_token_id", _U32, pad))
    kvs.append(("tokenizer.ggml.bos_token_id", _U32, pad))
    kvs.append(("tokenizer.ggml.add_bos_token", _BOOL, False))
    kvs.append(("tokenizer.chat_template", _STR, CHAT_TEMPLATE))
    n_kv = len(kvs) + 3
    w.u32(MAGIC)
    w.u32(3)
    w.u64(len(plan))
    w.u64(n_kv)
    for k, t, v in kvs:
        w.kv(k, t, v)
    w.arr("tokenizer.ggml.tokens", _STR, toks)
    w.arr("tokenizer.ggml.token_type", _I32, types)
    w.arr("tokenizer.ggml.merges", _STR, merges)
    off = 0
    offsets = []
    for name, shape, dt in plan:
        nbytes = int(np.prod(shape)) * _DTYPE_SIZE[dt]
        offsets.append(off)
        w.s(name)
        w.u32(len(shape))
        for dim in reversed(shape):
            w.u64(dim)
        w.u32(_DTYPE_CODE[dt])
        w.u64(off)
        off = _align(off + nbytes)
    pos = fh.tell()
    fh.write(b"\0" * (_align(pos) - pos))
    return fh.getvalue(), plan, offsets, fh.tell(), off


def _fill_jobs(cfg: Qwen3Shape, plan, offsets, data0: int) -> list[tuple]:
    """The random tensors as chunk jobs (file offset, seed, stream index,
    chunk index, elements, dtype, std); 2^22 elements per chunk."""
    jobs = []
    chunk_elems = 1 << 22
    for t_idx, ((name, shape, dt), o) in enumerate(zip(plan, offsets)):
        if _is_norm(name):
            continue
        n = int(np.prod(shape))
        esz = _DTYPE_SIZE[dt]
        for c_idx, start in enumerate(range(0, n, chunk_elems)):
            m = min(chunk_elems, n - start)
            jobs.append((data0 + o + start * esz, cfg.seed, rng_index(cfg, t_idx), c_idx, m, dt, cfg.std))
    return jobs


def _write_header(path: str, cfg: Qwen3Shape) -> list[tuple]:
    """Writes the header and the norm weights of the file at `path` (sized to
    its full length); returns the random-fill jobs."""
    head, plan, offsets, data0, total = _layout(cfg)
    with open(path, "wb") as fh:
        fh.write(head)
        for (name, shape, dt), o in zip(plan, offsets):
            if _is_norm(name):
                fh.seek(data0 + o)
                np.ones(int(np.prod(shape)), dtype="<f4").tofile(fh)
        fh.truncate(data0 + total)
    return _fill_jobs(cfg, plan, offsets, data0)


def _fill(path: str, jobs: list[tuple], threads: int | None = None) -> None:
    import concurrent.futures as cf

    fd = os.open(path, os.O_WRONLY)
    try:
        nthreads = threads or min(32, os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(max_workers=nthreads) as ex:
            for f in [ex.submit(_fill_chunk, fd, *j) for j in jobs]:
                f.result()
    finally:
        os.close(fd)


def write_qwen3_gguf(path: str | os.PathLike, cfg: Qwen3Shape, threads: int | None = None) -> str:
    """Write a seeded synthetic Qwen3 GGUF file; returns the path.

    Weights are N(0, cfg.std): tensor t is cut into chunks of 2^22 elements
    and chunk c is drawn from PCG64(SeedSequence([seed, t, c])), so the file
    is identical for any thread or process count. Norm weights are 1.0.
    """
    path = os.fspath(path)
    tmp = path + ".tmp"
    jobs = _write_header(tmp, cfg)
    _fill(tmp, jobs, threads)
    os.replace(tmp, path)
    return path


def ensure_gguf_ranks(path: str | os.PathLike, cfg: Qwen3Shape, rank: int, world: int, barrier) -> str:
    """ensure_gguf shared by `world` processes (one per GPU): rank 0 writes
    the header, every rank draws its share of the weight chunks, rank 0
    renames the finished file. `barrier()` synchronises the processes; every
    rank must call this with the same arguments."""
    path = os.fspath(path)
    tmp = path + ".ranks.tmp"
    exists = os.path.exists(path)
    barrier()
    if exists:
        return path
    if rank == 0:
        jobs = _write_header(tmp, cfg)
    else:
        _, plan, offsets, data0, _ = _layout(cfg)
        jobs = _fill_jobs(cfg, plan, offsets, data0)
    barrier()
    _fill(tmp, jobs[rank::world])
    barrier()
    if rank == 0:
        os.replace(tmp, path)
    barrier()
    return path


def ensure_gguf(path: str | os.PathLike, cfg: Qwen3Shape) -> str:
    """Write the file unless it is already there. The file appears atomically
    (written under a temporary name, then renamed), so processes that race to
    create it never read a partial file."""
    path = os.fspath(path)
    if not os.path.exists(path):
        tmp = f"{path}.tmp{os.getpid()}"
        try:
            write_qwen3_gguf(tmp, cfg)
            os.replace(tmp, path)
        finally:
            if os.path.exists(tmp):
                os.remove(tmp)
    return path


def random_prompt(n: int, vocab: int, seed: int) -> np.ndarray:
    """Prompt ids drawn like BaseModel::benchmark (src/base/model.cpp:189-193).

    std::mt19937(seed) feeding std::uniform_int_distribution<int>(0, V-1). For
    a 32-bit engine libstdc++ 13 maps each word w to [0, V) with Lemire's
    multiply-shift method (bits/uniform_int_dist.h, `_S_nd`): p = w * V;
    reject while the low 32 bits of p are below (2^32 - V) mod V; id = p >> 32.
    """
    words = _mt19937_words(seed)
    out = np.empty(n, dtype=np.uint32)
    thresh = ((1 << 32) - vocab) % vocab
    for i in range(n):
        prod = next(words) * vocab
        low = prod & 0xFFFFFFFF
        if low < vocab:
            while low < thresh:
                prod = next(words) * vocab
                low = prod & 0xFFFFFFFF
        out[i] = prod >> 32
    return out


def _mt19937_words(seed: int) -> Iterable[int]:
    """The 32-bit Mersenne Twister (std::mt19937) output stream."""
    mt = [0] * 624
    mt[0] = seed & 0xFFFFFFFF
    for i in range(1, 624):
        mt[i] = (1812433253 * (mt[i - 1] ^ (mt[i - 1] >> 30)) + i) & 0xFFFFFFFF
    idx = 624
    while True:
        if idx >= 624:
            for i in range(624):
                y = (mt[i] & 0x80000000) | (mt[(i + 1) % 624] & 0x7FFFFFFF)
                mt[i] = mt[(i + 397) % 624] ^ (y >> 1) ^ (0x9908B0DF if y & 1 else 0)
            idx = 0
        y = mt[idx]
        idx += 1
        y ^= y >> 11
        y ^= (y << 7) & 0x9D2C5680
        y ^= (y << 15) & 0xEFC60000
        y ^= y >> 18
        yield y & 0xFFFFFFFF
