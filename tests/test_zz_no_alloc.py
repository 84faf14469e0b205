"""The no-allocation attention entry point (mf_attn_decode_noalloc).

Callers that cannot allocate device memory (global-mode stream capture,
stream callbacks, memory owned by another runtime) use this variant: it takes
only inputs and outputs and keeps its scratch in a static device array. These
checks call it through the C ABI twice in a row and compare each result with
mf_attn_decode (caller workspace) within the attention tests' tolerance. The
file is named to run last, so a run stopping at its first failure has already
run everything else; it also passes on its own in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _desc(lib_mod, ptrs, S, H, Hkv, D, n_split, ws):
    from minfer_b200._lib import mf_attn_desc

    qkv, qn, kn, rope, kc, vc, st, out = ptrs
    return mf_attn_desc(qkv.data_ptr(), qn.data_ptr(), kn.data_ptr(), 1e-6, rope.data_ptr(), kc.data_ptr(),
                        vc.data_ptr(), S, st.data_ptr(), out.data_ptr(), H, Hkv, D, n_split,
                        ws.data_ptr() if ws is not None else None)


@pytest.mark.parametrize("H,Hkv,pos", [(32, 8, 4095), (16, 2, 300), (4, 2, 0)])
def test_noalloc_matches_workspace_variant(gpu, H, Hkv, pos):
    from minfer_b200 import ops
    from minfer_b200._lib import check, cuda_lib

    lib = cuda_lib()
    D, S = 128, 4160
    g = torch.Generator(device="cuda").manual_seed(H + pos)
    qkv = torch.randn((H + 2 * Hkv) * D, generator=g, device=gpu)
    qn = 1 + 0.1 * torch.randn(D, generator=g, device=gpu)
    kn = 1 + 0.1 * torch.randn(D, generator=g, device=gpu)
    kc0 = torch.randn(Hkv * S * D, generator=g, device=gpu)
    vc0 = torch.randn(Hkv * S * D, generator=g, device=gpu)
    rope = ops.rope_table(S, D, 1e6).to(gpu)
    st = torch.tensor([0, pos, 0, 0, 0, 0, 0, 0], dtype=torch.int32, device=gpu)
    n_split = ops.attn_default_split(Hkv, S)
    stream = ops._stream()

    # existing entry point, caller workspace
    kc, vc = kc0.clone(), vc0.clone()
    ref = torch.zeros(H * D, device=gpu)
    ws = torch.zeros(ops.attn_workspace_bytes(H, Hkv, D, n_split) // 4 + 1, dtype=torch.int32, device=gpu)
    d = _desc(ops, (qkv, qn, kn, rope, kc, vc, st, ref), S, H, Hkv, D, n_split, ws)
    check(lib.mf_attn_decode(C.byref(d), stream))
    torch.cuda.synchronize()
    ref_np = ref.cpu().numpy()
    ref_k = kc.view(Hkv, S, D)[:, pos].cpu().numpy()

    # new entry point, two calls in a row on fresh caches
    kc2, vc2 = kc0.clone(), vc0.clone()
    for call in range(2):
        out = torch.full((H * D,), float("nan"), device=gpu)
        d2 = _desc(ops, (qkv, qn, kn, rope, kc2, vc2, st, out), S, H, Hkv, D, n_split, None)
        check(lib.mf_attn_decode_noalloc(C.byref(d2), stream))
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.cpu().numpy(), ref_np, rtol=2e-5, atol=2e-5, err_msg=f"call {call}")
        np.testing.assert_allclose(kc2.view(Hkv, S, D)[:, pos].cpu().numpy(), ref_k, rtol=2e-6, atol=2e-6)


def test_noalloc_rejects_oversized_request(gpu):
    from minfer_b200 import ops
    from minfer_b200._lib import MF_E_UNSUPPORTED, cuda_lib

    lib = cuda_lib()
    H, Hkv, D, S = 64, 8, 128, 64
    t = torch.zeros(1 << 20, device=gpu)
    st = torch.tensor([0, 3, 0, 0, 0, 0, 0, 0], dtype=torch.int32, device=gpu)
    # 8 KV heads x 148 slices x 8 heads x 130 floats needs ~4.9 MB of scratch
    d = _desc(ops, (t, t, t, t, t, t, st, t), S, H, Hkv, D, 148, None)
    rc = lib.mf_attn_decode_noalloc(C.byref(d), ops._stream())
    assert rc == MF_E_UNSUPPORTED
    # the CUDA library's own message (the model library keeps a separate one)
    msg = C.create_string_buffer(512)
    lib.mf_last_error(msg, 512)
    assert b"MF_ATTN_NOALLOC_SCRATCH_BYTES" in msg.value
