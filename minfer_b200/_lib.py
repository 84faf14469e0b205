"""ctypes bindings of libmfcuda.so (include/minfer_cuda.h) and
libminfer_host.so (include/minfer_model.h).

The libraries are built in-tree (minfer_b200/lib). There is no fallback: if a
library is missing or fails to load, import of the op/model modules raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_DIR = Path(__file__).resolve().parent / "lib"
LIBMFCUDA = LIB_DIR / "libmfcuda.so"
LIBHOST = LIB_DIR / "libminfer_host.so"

MF_OK = 0
MF_E_INVALID = -1
MF_E_CUDA = -2
MF_E_OOM = -3
MF_E_TIMEOUT = -4
MF_E_UNSUPPORTED = -5
MF_E_STATE = -6
MF_E_IO = -7

MF_F32, MF_F16, MF_BF16 = 0, 1, 2
MF_TP_MAX = 8
MF_COMM_HANDLE_BYTES = 64
MF_STEP_RECORD_BYTES = 32
MF_STEP_FRAME = 4
MF_PREFILL_STORE, MF_PREFILL_RESID, MF_PREFILL_SWIGLU = 0, 1, 2
MF_FRAME_RECORD, MF_FRAME_REPLAY = 0, 1
MF_GEN_STOP_AT_EOS, MF_GEN_MARGINS, MF_GEN_TOKEN_PREFILL = 1, 2, 4

_STATUS = {
    MF_E_INVALID: "invalid argument",
    MF_E_CUDA: "CUDA error",
    MF_E_OOM: "out of memory",
    MF_E_TIMEOUT: "timeout",
    MF_E_UNSUPPORTED: "unsupported",
    MF_E_STATE: "bad state",
    MF_E_IO: "I/O error",
}


class MinferError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{_STATUS.get(code, code)}: {msg}")
        self.code = code


class mf_run_params(C.Structure):
    _fields_ = [("num_iters", C.c_size_t), ("max_seq_len", C.c_size_t), ("top_k", C.c_size_t),
                ("temp", C.c_float), ("top_p", C.c_float), ("min_p", C.c_float), ("penalty_pres", C.c_float),
                ("seed", C.c_int)]


class mf_model_info(C.Structure):
    _fields_ = [("vocab_size", C.c_size_t), ("max_seq_len", C.c_size_t),
                ("d_model", C.c_int), ("n_layers", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("d_head", C.c_int), ("d_ff", C.c_int), ("n_experts", C.c_int), ("n_active_experts", C.c_int),
                ("weight_dtype", C.c_int), ("untied_head", C.c_int), ("eos_token_id", C.c_uint32),
                ("rms_norm_eps", C.c_float), ("freq_base", C.c_float),
                ("read_bytes_logits", C.c_size_t), ("read_bytes_no_logits", C.c_size_t),
                ("kv_bytes_per_pos", C.c_size_t), ("tp_rank", C.c_int), ("tp_size", C.c_int),
                ("expert_parallel", C.c_int)]


class mf_gen_stats(C.Structure):
    _fields_ = [("num_tokens_gen", C.c_int), ("ttft", C.c_float), ("throughput", C.c_float),
                ("prefill_time", C.c_float), ("bandwidth", C.c_float), ("decode_seconds", C.c_double),
                ("bytes_read", C.c_double)]


class mf_attn_desc(C.Structure):
    _fields_ = [("qkv", C.c_void_p), ("q_norm_w", C.c_void_p), ("k_norm_w", C.c_void_p), ("eps", C.c_float),
                ("rope_table", C.c_void_p), ("k_cache", C.c_void_p), ("v_cache", C.c_void_p), ("max_seq", C.c_int),
                ("step_state", C.c_void_p), ("out", C.c_void_p), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("d_head", C.c_int), ("n_split", C.c_int), ("workspace", C.c_void_p), ("kv_dtype", C.c_int)]


P = C.c_void_p
I = C.c_int
U32 = C.c_uint32
SZ = C.c_size_t
F = C.c_float

# name -> (restype, argtypes). Every function of the two public headers.
CUDA_API = {
    "mf_init": (I, [I, P]),
    "mf_shutdown": (I, []),
    "mf_device_count": (I, [P]),
    "mf_decode_status": (I, [I, P, I]),
    "mf_last_error": (I, [C.c_char_p, SZ]),
    "mf_upload": (I, [P, SZ, I, P]),
    "mf_alloc": (I, [SZ, I, P]),
    "mf_release": (None, [P]),
    "mf_ptr": (P, [P]),
    "mf_size": (SZ, [P]),
    "mf_read": (I, [P, SZ, P, SZ]),
    "mf_write": (I, [P, SZ, P, SZ]),
    "mf_write_2d": (I, [P, SZ, SZ, P, SZ, SZ, SZ]),
    "mf_copy": (I, [P, SZ, P, SZ, SZ]),
    "mf_host_alloc": (I, [SZ, P]),
    "mf_host_free": (None, [P]),
    "mf_copy_to_host_async": (I, [P, P, SZ, P]),
    "mf_begin_frame": (I, [I, I]),
    "mf_begin_frame_ex": (I, [I, I, I]),
    "mf_end_frame": (I, [I]),
    "mf_end_frame_async": (I, [I]),
    "mf_abort_frame": (I, [I]),
    "mf_reset_frames": (I, [I]),
    "mf_drop_frames": (I, [I, I, I]),
    "mf_sync": (I, [I]),
    "mf_stream": (P, [I]),
    "mf_timer_start": (I, [I]),
    "mf_timer_stop": (I, [I, P]),
    "mf_step_state": (I, [I, P, P]),
    "mf_embed_step": (I, [P, P, I, I, I, P, P]),
    "mf_rope_table": (I, [P, I, I, F]),
    "mf_rmsnorm_matmul": (I, [P, P, P, F, P, I, I, I, P]),
    "mf_matmul_residual": (I, [P, P, P, I, I, I, P]),
    "mf_swiglu_matmul": (I, [P, P, P, F, P, I, I, I, P]),
    "mf_attn_workspace_bytes": (SZ, [I, I, I, I]),
    "mf_attn_default_split": (I, [I, I]),
    "mf_attn_decode": (I, [P, P]),
    "mf_attn_decode_noalloc": (I, [P, P]),
    "mf_router_topk": (I, [P, P, P, P, P, F, P, I, I, I, P]),
    "mf_moe_swiglu": (I, [P, P, P, F, P, I, P, I, I, I, P]),
    "mf_moe_down_residual": (I, [P, P, P, I, P, P, I, I, I, P]),
    "mf_moe_ffn": (I, [P, P, P, F, P, P, P, I, P, P, P, I, I, I, I, P]),
    "mf_lm_head_workspace_bytes": (SZ, []),
    "mf_lm_head": (I, [P, P, P, F, P, I, I, I, I, P, P, P]),
    "mf_comm_create": (I, [I, I, I, I, I, P]),
    "mf_comm_create_ex": (I, [I, I, I, I, I, SZ, P]),
    "mf_comm_handle": (I, [P, P, SZ]),
    "mf_comm_connect": (I, [P, P, SZ]),
    "mf_comm_status": (I, [P, P, I]),
    "mf_comm_gather_ptr": (I, [P, P]),
    "mf_comm_bulk_ptr": (I, [P, I, P]),
    "mf_bulk_allreduce": (I, [P, SZ, P, I, C.c_ulonglong, P]),
    "mf_comm_destroy": (None, [P]),
    "mf_matmul_push": (I, [P, P, I, I, I, P, I, P, P]),
    "mf_allreduce_rmsnorm_matmul": (I, [P, P, P, P, F, P, I, I, I, P, I, P, P]),
    "mf_allreduce_swiglu_matmul": (I, [P, P, P, P, F, P, I, I, I, P, I, P, P]),
    "mf_allreduce_lm_head": (I, [P, P, P, P, F, P, I, I, I, I, P, P, I, P, I, P]),
    "mf_allreduce": (I, [P, P, P, I, P, I, P, P]),
    "mf_allreduce_router_topk": (I, [P, P, P, P, P, P, F, P, I, I, I, P, I, P, P]),
    "mf_moe_swiglu_ep": (I, [P, P, P, F, P, I, P, I, I, I, I, I, P]),
    "mf_moe_down_push": (I, [P, P, I, P, P, I, I, I, I, I, P, I, P, P]),
    "mf_prefill_gemm": (I, [P, I, P, P, P, I, I, I, I, P, P, P]),
    "mf_prefill_gemm_grouped": (I, [P, I, P, P, P, I, I, I, I, P, P, I, P, P, P]),
    "mf_prefill_moe_route": (I, [P, P, P, P, I, I, I, I, P]),
    "mf_prefill_moe_group": (I, [P, I, I, I, I, P, P, P, P]),
    "mf_prefill_moe_gather": (I, [P, P, P, P, I, I, I, P]),
    "mf_prefill_moe_combine": (I, [P, P, P, P, P, I, I, I, P]),
    "mf_prefill_norm_split": (I, [P, P, P, P, P, F, I, I, P]),
    "mf_prefill_split": (I, [P, P, P, SZ, P]),
    "mf_prefill_swiglu_split": (I, [P, P, P, I, I, P]),
    "mf_prefill_embed": (I, [P, P, I, I, I, P, I, P]),
    "mf_prefill_qkv_post": (I, [P, P, P, P, P, P, F, P, I, I, I, I, I, I, I, P]),
    "mf_prefill_attention": (I, [P, P, P, P, P, I, I, I, I, I, I, I, P]),
    "mf_prefill_attention_scratch": (I, [I, I, I, I, P]),
    "mf_prefill_attention_tc": (I, [P, P, P, P, P, I, I, I, I, I, I, P, SZ, I, P]),
    "mf_prefill_status": (I, [P, I]),
    "mf_topk_workspace_bytes": (SZ, [I, I]),
    "mf_topk": (I, [P, I, I, P, P, P, SZ, P]),
    "mf_sample_step": (I, [P, P, I, F, F, F, P, I, P, P, P, P]),
    "mf_matmul": (I, [P, P, P, I, SZ, I, I, P]),
    "mf_rmsnorm": (I, [P, P, P, I, F, I, P]),
    "mf_softmax": (I, [P, P, I, I, P]),
    "mf_silu": (I, [P, P, I, P]),
    "mf_neox_rope": (I, [P, P, I, I, I, F, I, P]),
    "mf_il_rope": (I, [P, P, I, I, I, F, I, P]),
    "mf_attn": (I, [P, P, P, P, P, I, I, I, P]),
    "mf_route": (I, [P, P, P, P, P, I, I, I, P]),
    "mf_embed": (I, [P, P, I, U32, I, P]),
    "mf_argmax": (I, [P, I, P, P]),
}

HOST_API = {
    "mf_host_last_error": (I, [C.c_char_p, SZ]),
    "mf_model_load": (I, [C.c_char_p, P, I, P]),
    "mf_model_to_cuda": (I, [P]),
    "mf_model_set_kv_dtype": (I, [P, I]),
    "mf_model_load_tp": (I, [C.c_char_p, P, I, I, I, P]),
    "mf_model_prefill": (I, [P, P, SZ, I, I, I]),
    "mf_model_comm_handle": (I, [P, P, SZ]),
    "mf_model_comm_connect": (I, [P, P, SZ]),
    "mf_model_comm_status": (I, [P, P]),
    "mf_model_info_get": (I, [P, P]),
    "mf_model_free": (None, [P]),
    "mf_model_forward": (I, [P, U32, I, I, I]),
    "mf_model_logits": (I, [P, P, SZ]),
    "mf_model_argmax": (I, [P, P]),
    "mf_model_generate": (I, [P, P, SZ, SZ, I, P, P, P, P, P]),
    "mf_model_generate_logits": (I, [P, P, SZ, SZ, I, P, P, P, P, P, P, SZ, P]),
    "mf_model_decode_chained": (I, [P, U32, I, I, P]),
    "mf_model_benchmark": (I, [P, I, P]),
    "mf_model_reset_sampler": (I, [P]),
    "mf_model_experts": (I, [P, I, P, P]),
    "mf_model_prefill_experts": (I, [P, I, P, P, I]),
    "mf_model_kv": (I, [P, I, P, P, I]),
    "mf_model_x": (I, [P, P]),
    "mf_random_prompt": (I, [I, U32, SZ, P]),
    "mf_tokenizer_load": (I, [C.c_char_p, P]),
    "mf_tokenizer_create": (I, [P, P, P, SZ, P, P, SZ, C.c_char_p, U32, U32, P]),
    "mf_tokenizer_free": (None, [P]),
    "mf_tokenizer_info": (I, [P, P, P, P]),
    "mf_tokenizer_encode": (I, [P, C.c_char_p, SZ, P, SZ, P]),
    "mf_tokenizer_decode": (I, [P, P, SZ, C.c_char_p, SZ, P]),
    "mf_tokenizer_pre_split": (I, [P, C.c_char_p, SZ, P, SZ, P]),
    "mf_tokenizer_apply_chat_template": (I, [P, C.c_char_p, C.c_char_p, I, C.c_char_p, SZ, P]),
    "mf_sample": (I, [P, SZ, P, P, SZ, SZ, P]),
    "mf_sample_candidates": (I, [P, SZ, P, SZ, P]),
}

_cuda = None
_host = None


def _bind(lib: C.CDLL, api: dict) -> None:
    for name, (res, args) in api.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def cuda_lib() -> C.CDLL:
    """libmfcuda.so, loaded once; raises if it was not built."""
    global _cuda
    if _cuda is None:
        if not LIBMFCUDA.exists():
            raise ImportError(f"{LIBMFCUDA} is missing: build it with `python -m minfer_b200.build`")
        lib = C.CDLL(str(LIBMFCUDA), mode=os.RTLD_NOW | os.RTLD_GLOBAL)
        _bind(lib, CUDA_API)
        _cuda = lib
    return _cuda


def host_lib() -> C.CDLL:
    global _host
    if _host is None:
        cuda_lib()
        if not LIBHOST.exists():
            raise ImportError(f"{LIBHOST} is missing: build it with `python -m minfer_b200.build`")
        lib = C.CDLL(str(LIBHOST), mode=os.RTLD_NOW | os.RTLD_GLOBAL)
        _bind(lib, HOST_API)
        _host = lib
    return _host


def last_error() -> str:
    buf = C.create_string_buffer(512)
    if _host is not None:
        _host.mf_host_last_error(buf, 512)
    else:
        cuda_lib().mf_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(rc: int) -> int:
    if rc is not None and rc < 0:
        raise MinferError(rc, last_error())
    return rc
