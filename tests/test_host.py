"""Host-side pieces on the CPU: the C-ABI libraries load and export every
symbol their headers declare; the GGUF reader accepts the synthetic models
and rejects malformed files with a status and a message; the prompt-id draw,
the RoPE table and the sampler agree with the oracle. No kernel is launched.
"""
import ctypes as C
import re
import struct
from pathlib import Path

import numpy as np
import pytest

from conftest import TINY, tiny_model
from minfer_b200._lib import (HOST_API, CUDA_API, MF_E_INVALID, MF_E_UNSUPPORTED, MF_OK, cuda_lib, host_lib,
                              last_error, mf_model_info, mf_run_params)
from minfer_b200.gguf_synth import Qwen3Shape, random_prompt, write_qwen3_gguf
from oracle.oracle_py import PortModel, PortOps

ROOT = Path(__file__).resolve().parent.parent


def header_functions(name: str) -> set[str]:
    text = (ROOT / "include" / name).read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"^\s*(?:int|void\*?|size_t)\s+\*?(mf_\w+)\s*\(", text, flags=re.M))


def test_every_declared_symbol_is_exported():
    cuda, host = cuda_lib(), host_lib()
    for hdr, lib in (("minfer_cuda.h", cuda), ("minfer_model.h", host)):
        names = header_functions(hdr)
        assert len(names) > 10
        for n in sorted(names):
            assert hasattr(lib, n), f"{n} declared in {hdr} but not exported"
    # the ctypes prototype table covers the headers exactly
    assert header_functions("minfer_cuda.h") == set(CUDA_API)
    assert header_functions("minfer_model.h") == set(HOST_API)


def load(path, **kw):
    rp = mf_run_params(kw.get("num_iters", 8), kw.get("max_seq", 64), kw.get("top_k", 1), kw.get("temp", 0.0),
                       kw.get("top_p", 1.0), 0.0, 0.0, kw.get("seed", 0))
    m = C.c_void_p()
    rc = host_lib().mf_model_load(str(path).encode(), C.byref(rp), 0, C.byref(m))
    return rc, m


@pytest.mark.parametrize("name", list(TINY))
def test_gguf_config(name):
    rc, m = load(tiny_model(name))
    assert rc == MF_OK, last_error()
    info = mf_model_info()
    assert host_lib().mf_model_info_get(m, C.byref(info)) == MF_OK
    cfg = TINY[name]
    assert (info.d_model, info.n_layers, info.n_heads, info.n_kv_heads, info.d_head, info.d_ff) == (
        cfg.d_model, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.d_head, cfg.d_ff)
    assert (info.n_experts, info.n_active_experts, info.vocab_size) == (cfg.n_experts, cfg.n_active, cfg.vocab)
    assert info.untied_head == (0 if cfg.tied else 1)
    assert info.weight_dtype == {"f32": 0, "f16": 1, "bf16": 2}[cfg.dtype]
    assert abs(info.freq_base - 1e6) < 1 and abs(info.rms_norm_eps - 1e-6) < 1e-12
    host_lib().mf_model_free(m)


def _corrupt(tmp_path, fn, data: bytes) -> Path:
    p = tmp_path / fn
    p.write_bytes(data)
    return p


def test_gguf_rejects_malformed(tmp_path):
    good = Path(tiny_model("tiny-bf16")).read_bytes()
    cases = {
        "bad_magic.gguf": b"XXXX" + good[4:],
        "v2.gguf": good[:4] + struct.pack("<I", 2) + good[8:],
        "truncated.gguf": good[:4096],
        "empty.gguf": b"",
        "zero_tensors.gguf": good[:8] + struct.pack("<Q", 0) + good[16:],
    }
    for fn, data in cases.items():
        rc, _ = load(_corrupt(tmp_path, fn, data))
        assert rc != MF_OK, fn
        assert last_error(), fn
    rc, _ = load(tmp_path / "missing.gguf")
    assert rc != MF_OK and "missing.gguf" in last_error()


def test_gguf_rejects_bad_run_params(tmp_path):
    rc, _ = load(tiny_model("tiny-bf16"), max_seq=10 ** 9)  # beyond context_length
    assert rc != MF_OK and "max_seq_len" in last_error()


def test_gguf_rejects_unsupported_dtype(tmp_path):
    cfg = Qwen3Shape(1, 64, 2, 1, 128, 64, 300, "bf16", True, seed=1)
    p = write_qwen3_gguf(tmp_path / "m.gguf", cfg)
    data = bytearray(Path(p).read_bytes())
    # the first tensor info's type field (BF16 = 30) -> Q4_0 (2)
    idx = data.find(b"token_embd.weight")
    off = idx + len(b"token_embd.weight") + 4 + 2 * 8
    assert struct.unpack_from("<I", data, off)[0] == 30
    struct.pack_into("<I", data, off, 2)
    rc, _ = load(_corrupt(tmp_path, "q4.gguf", bytes(data)))
    assert rc != MF_OK and "unsupported type" in last_error()


def test_random_prompt_matches_benchmark_draw():
    # C++ std::mt19937 + uniform_int_distribution (host library) vs the Python restatement
    out = np.zeros(2000, np.uint32)
    assert host_lib().mf_random_prompt(30, 151936, 2000, out.ctypes.data) == MF_OK
    assert np.array_equal(out, random_prompt(2000, 151936, 30))
    out = np.zeros(500, np.uint32)
    host_lib().mf_random_prompt(7, 1000, 500, out.ctypes.data)
    assert np.array_equal(out, random_prompt(500, 1000, 7))


def test_rope_table_matches_oracle():
    tab = np.zeros((64, 64, 2), np.float32)
    assert cuda_lib().mf_rope_table(tab.ctypes.data, 64, 128, 1e6) == MF_OK
    po = PortOps()
    for pos in (0, 1, 63):
        for i in (0, 17, 63):
            e = np.zeros(128, np.float32)
            e[i] = 1
            o = po.rope(e, 0, 128, 128, 1e6, pos)
            assert o[i] == tab[pos, i, 0] and o[i + 64] == tab[pos, i, 1]


@pytest.mark.parametrize("temp,top_k,top_p,min_p,pres", [(0.0, 1, 1.0, 0.0, 0.0), (0.7, 20, 0.9, 0.0, 0.0),
                                                         (0.6, 20, 0.95, 0.0, 1.5), (1.0, 50, 1.0, 0.05, 0.0)])
def test_sampler_matches_oracle(temp, top_k, top_p, min_p, pres):
    V = TINY["tiny-bf16"].vocab
    rng = np.random.default_rng(int(temp * 10) + top_k)
    logits = (rng.standard_normal(V) * 2).astype(np.float32)
    logits[5] = logits[6] = logits.max() + 1  # a tie at the top
    seen = np.array([5, 9, 100, 200], np.uint32)
    rp = mf_run_params(0, 64, top_k, temp, top_p, min_p, pres, 42)
    n = 64
    out = np.zeros(n, np.uint32)
    assert host_lib().mf_sample(logits.ctypes.data, V, C.byref(rp), seen.ctypes.data, seen.size, n,
                                out.ctypes.data) == MF_OK
    pm = PortModel(tiny_model("tiny-bf16"), max_seq=8, top_k=top_k, temp=temp, top_p=top_p, min_p=min_p, pres=pres,
                   seed=42)
    for s in seen:
        pm.add_token(int(s))
    ref = [pm.sample(logits) for _ in range(n)]
    assert out.tolist() == ref
    if temp == 0.0:
        assert set(ref) == {5}  # first maximum


@pytest.mark.parametrize("case", ["inside", "boundary", "none"])
def test_candidate_sampling_with_tied_logits(case):
    """generate() samples from the device's top-k list (equal logits lower id
    first) only when no two of its top_k + 1 values are equal; otherwise the
    whole-vocabulary sampler decides. Either way the ids equal the reference
    sampler's (nth_element + sort) on the same logits."""
    V, k = 1024, 20
    rng = np.random.default_rng({"inside": 1, "boundary": 2, "none": 3}[case])
    logits = (rng.standard_normal(V) * 2).astype(np.float32)
    order = np.argsort(-logits, kind="stable")
    if case == "inside":  # ties among the top-k: ids 900 and 3 share the 2nd value
        logits[900] = logits[3] = logits[order[1]]
    elif case == "boundary":  # the k-th and (k+1)-th logits are equal
        logits[order[k]] = logits[order[k - 1]]
    rp = mf_run_params(0, 64, k, 0.9, 0.95, 0.0, 0.0, 42)
    n = 256
    got = np.zeros(n, np.uint32)
    assert host_lib().mf_sample_candidates(logits.ctypes.data, V, C.byref(rp), n, got.ctypes.data) == MF_OK
    ref = np.zeros(n, np.uint32)
    assert host_lib().mf_sample(logits.ctypes.data, V, C.byref(rp), None, 0, n, ref.ctypes.data) == MF_OK
    assert got.tolist() == ref.tolist()


def test_sampling_rule_rebuilds_the_reference_draw():
    """The sampling distribution the flip rule of the GPU tests rebuilds
    (tests/sampling_rule.py), with the reference's random numbers
    (oracle uniform_draws), picks exactly the reference sampler's ids."""
    from oracle.oracle_py import uniform_draws
    from sampling_rule import pick, sampling_cdf

    V, n = 4096, 200
    for seed, (temp, top_k, top_p, min_p) in enumerate([(0.7, 20, 0.9, 0.0), (1.0, 40, 0.95, 0.05), (0.5, 5, 1.0, 0.0)]):
        logits = (np.random.default_rng(seed).standard_normal(V) * 2).astype(np.float32)
        rp = mf_run_params(0, 64, top_k, temp, top_p, min_p, 0.0, 42 + seed)
        ref = np.zeros(n, np.uint32)
        assert host_lib().mf_sample(logits.ctypes.data, V, C.byref(rp), None, 0, n, ref.ctypes.data) == MF_OK
        order = np.argsort(-logits, kind="stable")[:top_k]
        cdf, _, _ = sampling_cdf(logits[order], temp, top_p, min_p)
        r = uniform_draws(42 + seed, n)
        assert [pick(order, cdf, x) for x in r] == ref.tolist()


def test_prefix_gguf_shares_the_full_models_weights(tmp_path):
    """A depth-reduced prefix file holds the same embedding, layers and lm_head
    as the first layers of the full model (same random streams)."""
    from minfer_b200.gguf_synth import Qwen3Shape, write_qwen3_gguf

    full = Qwen3Shape(4, 64, 2, 1, 32, 64, 300, "bf16", False, seed=5)
    a = write_qwen3_gguf(tmp_path / "full.gguf", full)
    b = write_qwen3_gguf(tmp_path / "pre.gguf", full.prefix(2))

    # tensor data is the file's tail, tensors in plan order at ALIGN-aligned offsets
    def raw(path, cfg):
        from minfer_b200.gguf_synth import ALIGN, _DTYPE_SIZE, tensor_plan
        data = open(path, "rb").read()
        plan = tensor_plan(cfg)
        sizes = [int(np.prod(sh)) * _DTYPE_SIZE[dt] for _, sh, dt in plan]
        tail = 0
        for sz in sizes:
            tail = (tail + sz + ALIGN - 1) // ALIGN * ALIGN
        data0 = len(data) - tail
        out, off = {}, 0
        for (name, _, _), sz in zip(plan, sizes):
            out[name] = data[data0 + off:data0 + off + sz]
            off = (off + sz + ALIGN - 1) // ALIGN * ALIGN
        return out

    ra, rb = raw(a, full), raw(b, full.prefix(2))
    for name in rb:
        assert ra[name] == rb[name], name
    assert "blk.3.attn_q.weight" in ra and "blk.3.attn_q.weight" not in rb


def test_sampler_rejects_bad_params():
    logits = np.zeros(16, np.float32)
    out = np.zeros(1, np.uint32)
    rp = mf_run_params(0, 8, 0, 0.7, 0.9, 0.0, 0.0, 1)  # top_k = 0
    assert host_lib().mf_sample(logits.ctypes.data, 16, C.byref(rp), None, 0, 1, out.ctypes.data) == MF_E_INVALID


def test_ops_validate_before_touching_the_device():
    lib = cuda_lib()
    # null pointers and bad sizes are rejected on the host, no GPU needed
    assert lib.mf_matmul(None, None, None, 2, 0, 16, 16, None) == MF_E_INVALID
    assert lib.mf_rmsnorm(None, None, None, 0, 1e-6, 1, None) == MF_E_INVALID
    assert lib.mf_attn_decode(None, None) == MF_E_INVALID
    assert lib.mf_attn_decode_noalloc(None, None) == MF_E_INVALID
    # tensor-core prefill attention: scratch size and alignment are checked before any device call
    need = C.c_size_t()
    assert lib.mf_prefill_attention_scratch(100, 140, 32, 8, C.byref(need)) == MF_OK
    ld = 192  # 140 keys rounded up to 64
    assert need.value == 4 * 8 * ld * 128 * 2  # K fp16 hi/lo and V^T bf16 hi/lo
    assert lib.mf_prefill_attention_scratch(100, 99, 32, 8, C.byref(need)) == MF_E_INVALID
    fake = C.c_void_p(1 << 20)
    args = (fake, fake, fake, fake, fake, 256, 100, 40, 32, 8, 128)  # 40 + 100 = 140 keys
    assert lib.mf_prefill_attention_tc(*args, fake, need.value - 1, 0, None) == MF_E_INVALID
    msg = C.create_string_buffer(256)
    lib.mf_last_error(msg, 256)
    assert b"scratch too small" in msg.value
    # device top-k: k limits and workspace size are checked on the host
    assert lib.mf_topk_workspace_bytes(151936, 20) == 256 + 149 * 20 * 8
    assert lib.mf_topk(fake, 151936, 65, fake, fake, fake, 1 << 20, None) == MF_E_INVALID
    assert lib.mf_topk(fake, 10, 20, fake, fake, fake, 1 << 20, None) == MF_E_INVALID
    assert lib.mf_topk(fake, 151936, 20, fake, fake, fake, 100, None) == MF_E_INVALID
    # bulk exchange: arguments checked before any device work
    assert lib.mf_bulk_allreduce(None, 16, None, 0, 1, None) == MF_E_INVALID
    assert lib.mf_bulk_allreduce(fake, 16, None, 2, 1, None) == MF_E_INVALID
    assert lib.mf_comm_bulk_ptr(None, 0, C.byref(C.c_void_p())) == MF_E_INVALID
    assert lib.mf_prefill_attention_tc(*args, C.c_void_p((1 << 20) + 16), need.value, 0, None) == MF_E_INVALID
    assert lib.mf_prefill_attention_tc(*args[:6], 300, *args[7:], fake, need.value, 0, None) == MF_E_INVALID
    assert lib.mf_prefill_attention_tc(*args, fake, need.value, 1, None) == MF_E_UNSUPPORTED  # f16 cache
    assert lib.mf_lm_head(None, None, None, 1e-6, None, 2, 10, 16, 0, None, None, None) == MF_E_INVALID
