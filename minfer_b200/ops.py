"""The reference's CPU op interface (include/minfer/ops/kernels.hpp:13-32) and the
fused token-loop ops, on CUDA tensors, through libmfcuda's C ABI.

Arguments follow the reference's names and meaning (`out` first, then
inputs); tensors must be contiguous CUDA tensors (activations fp32, weights
fp32 / fp16 / bf16 — bf16 may also be passed as raw uint16 bit patterns).
Every call raises MinferError on a non-zero status.
"""
from __future__ import annotations

import ctypes as C

import torch

from ._lib import MF_BF16, MF_F16, MF_F32, check, cuda_lib, mf_attn_desc

_lib = cuda_lib()


def _ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    return t.data_ptr()


_CUDA_STREAM_LEGACY = 1  # cudaStreamLegacy: the C ABI reads a NULL stream as "manager stream"


def _stream() -> int:
    """torch's current stream as a cudaStream_t for the C ABI."""
    s = torch.cuda.current_stream().cuda_stream
    return s if s else _CUDA_STREAM_LEGACY


def dtype_code(w: torch.Tensor, dtype: str | None = None) -> int:
    if dtype is not None:
        return {"f32": MF_F32, "f16": MF_F16, "bf16": MF_BF16}[dtype]
    if w.dtype == torch.float32:
        return MF_F32
    if w.dtype == torch.float16:
        return MF_F16
    if w.dtype in (torch.bfloat16, torch.uint16, torch.int16):
        return MF_BF16
    raise ValueError(f"unsupported weight dtype {w.dtype}")


# ---------------------------------------------------------------- single ops

def matmul(out, x, weight, offset: int, d_out: int, d_in: int, dtype: str | None = None):
    """kernels.hpp `matmul`: out[i] = sum_j W[offset + i*d_in + j] * x[j]."""
    check(_lib.mf_matmul(_ptr(out), _ptr(x), _ptr(weight), dtype_code(weight, dtype), offset, d_out, d_in,
                         _stream()))


def rmsnorm(out, x, weight, dim: int, eps: float, n_rows: int = 1):
    check(_lib.mf_rmsnorm(_ptr(out), _ptr(x), _ptr(weight), dim, eps, n_rows, _stream()))


def softmax(out, x, size: int, n_rows: int = 1):
    check(_lib.mf_softmax(_ptr(out), _ptr(x), size, n_rows, _stream()))


def silu(out, x, n: int):
    check(_lib.mf_silu(_ptr(out), _ptr(x), n, _stream()))


def neox_rope(out, x, head_idx: int, d_head: int, d_rotary: int, freq_base: float, pos: int):
    check(_lib.mf_neox_rope(_ptr(out), _ptr(x), head_idx, d_head, d_rotary, freq_base, pos, _stream()))


def il_rope(out, x, head_idx: int, d_head: int, d_rotary: int, freq_base: float, pos: int):
    check(_lib.mf_il_rope(_ptr(out), _ptr(x), head_idx, d_head, d_rotary, freq_base, pos, _stream()))


def attn(att_scores, att_out, q_head, kh, vh, seq_len: int, d_head: int, kv_dim: int):
    check(_lib.mf_attn(_ptr(att_scores), _ptr(att_out), _ptr(q_head), _ptr(kh), _ptr(vh), seq_len, d_head, kv_dim,
                       _stream()))


def route(x_norm, active_experts, active_experts_weights, moe_scores, w_router, d_model: int, n_experts: int,
          n_active: int):
    check(_lib.mf_route(_ptr(x_norm), _ptr(active_experts), _ptr(active_experts_weights), _ptr(moe_scores),
                        _ptr(w_router), d_model, n_experts, n_active, _stream()))


def embed(out, weight, token_id: int, d_in: int, dtype: str | None = None):
    check(_lib.mf_embed(_ptr(out), _ptr(weight), dtype_code(weight, dtype), token_id, d_in, _stream()))


def argmax(logits, n: int, out):
    check(_lib.mf_argmax(_ptr(logits), n, _ptr(out), _stream()))


# ---------------------------------------------------------------- fused ops

def rope_table(n_pos: int, d_rot: int, base: float) -> torch.Tensor:
    """[n_pos, d_rot/2, 2] (cos, sin) in float (host tensor)."""
    out = torch.empty(n_pos, d_rot // 2, 2, dtype=torch.float32)
    check(_lib.mf_rope_table(C.c_void_p(out.data_ptr()), n_pos, d_rot, base))
    return out


def embed_step(x, emb, vocab: int, d_model: int, step_state, dtype: str | None = None):
    check(_lib.mf_embed_step(_ptr(x), _ptr(emb), dtype_code(emb, dtype), vocab, d_model, _ptr(step_state),
                             _stream()))


def rmsnorm_matmul(y, x, norm_w, eps: float, w, d_out: int, d_in: int, dtype: str | None = None):
    check(_lib.mf_rmsnorm_matmul(_ptr(y), _ptr(x), _ptr(norm_w), eps, _ptr(w), dtype_code(w, dtype), d_out, d_in,
                                 _stream()))


def matmul_residual(x, a, w, d_out: int, d_in: int, dtype: str | None = None):
    check(_lib.mf_matmul_residual(_ptr(x), _ptr(a), _ptr(w), dtype_code(w, dtype), d_out, d_in, _stream()))


def swiglu_matmul(h, x, norm_w, eps: float, w_gate_up, d_ff: int, d_in: int, dtype: str | None = None):
    check(_lib.mf_swiglu_matmul(_ptr(h), _ptr(x), _ptr(norm_w), eps, _ptr(w_gate_up), dtype_code(w_gate_up, dtype),
                                d_ff, d_in, _stream()))


def attn_workspace_bytes(n_heads: int, n_kv_heads: int, d_head: int, n_split: int) -> int:
    return int(_lib.mf_attn_workspace_bytes(n_heads, n_kv_heads, d_head, n_split))


def attn_default_split(n_kv_heads: int, max_seq: int) -> int:
    return int(_lib.mf_attn_default_split(n_kv_heads, max_seq))


def attn_decode(qkv, q_norm_w, k_norm_w, eps: float, rope_table, k_cache, v_cache, max_seq: int, step_state, out,
                n_heads: int, n_kv_heads: int, d_head: int, n_split: int, workspace):
    """The cache element type follows k_cache's dtype (float32 or bfloat16)."""
    d = mf_attn_desc(_ptr(qkv), _ptr(q_norm_w), _ptr(k_norm_w), eps, _ptr(rope_table), _ptr(k_cache), _ptr(v_cache),
                     max_seq, _ptr(step_state), _ptr(out), n_heads, n_kv_heads, d_head, n_split, _ptr(workspace),
                     dtype_code(k_cache))
    check(_lib.mf_attn_decode(C.byref(d), _stream()))


def router_topk(ids, weights, scores, x, norm_w, eps: float, w_router, d_model: int, n_experts: int, k: int):
    check(_lib.mf_router_topk(_ptr(ids), _ptr(weights), _ptr(scores), _ptr(x), _ptr(norm_w), eps, _ptr(w_router),
                              d_model, n_experts, k, _stream()))


def moe_swiglu(h, x, norm_w, eps: float, w_gate_up_exps, ids, k: int, d_ff: int, d_in: int,
               dtype: str | None = None):
    check(_lib.mf_moe_swiglu(_ptr(h), _ptr(x), _ptr(norm_w), eps, _ptr(w_gate_up_exps),
                             dtype_code(w_gate_up_exps, dtype), _ptr(ids), k, d_ff, d_in, _stream()))


def moe_down_residual(x, h, w_down_exps, ids, weights, k: int, d_model: int, d_ff: int, dtype: str | None = None):
    check(_lib.mf_moe_down_residual(_ptr(x), _ptr(h), _ptr(w_down_exps), dtype_code(w_down_exps, dtype), _ptr(ids),
                                    _ptr(weights), k, d_model, d_ff, _stream()))


def moe_ffn(x, h, norm_w, eps: float, w_router, w_gate_up_exps, w_down_exps, scores, ids, weights, d_model: int,
            d_ff: int, n_experts: int, k: int, dtype: str | None = None):
    """router_topk + moe_swiglu + moe_down_residual as one launch chain."""
    check(_lib.mf_moe_ffn(_ptr(x), _ptr(h), _ptr(norm_w), eps, _ptr(w_router), _ptr(w_gate_up_exps),
                          _ptr(w_down_exps), dtype_code(w_gate_up_exps, dtype), _ptr(scores), _ptr(ids), _ptr(weights),
                          d_model, d_ff, n_experts, k, _stream()))


def lm_head_workspace_bytes() -> int:
    return int(_lib.mf_lm_head_workspace_bytes())


def lm_head(logits, x, norm_w, eps: float, w, vocab: int, d_model: int, step_state=None, workspace=None,
            vocab_offset: int = 0, dtype: str | None = None):
    check(_lib.mf_lm_head(_ptr(logits), _ptr(x), _ptr(norm_w), eps, _ptr(w), dtype_code(w, dtype), vocab, d_model,
                          vocab_offset, _ptr(step_state), _ptr(workspace), _stream()))
