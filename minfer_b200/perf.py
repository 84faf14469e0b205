"""Single-kernel timing of the token-loop ops on synthetic operands.

    python -m minfer_b200.perf gemv --rows 24576 --k 4096 --mode swiglu
    python -m minfer_b200.perf attn --hq 32 --hkv 8 --ctx 4096
    python -m minfer_b200.perf gemm --m 4096 --n 24576 --k 4096 --mode swiglu
    python -m minfer_b200.perf pattn --p 4096 --pos0 0 --hq 32 --hkv 8 --kernel tc

Prints one JSON line per case: average device time per launch (CUDA events
around a CUDA-graph replay of `--iters` launches on torch's stream, after
warm-up launches) and the algorithmic bytes per launch divided by that time. Operand sets larger than L2 are rotated between launches
(`--copies`) so every launch streams from HBM.
"""
from __future__ import annotations

import argparse
import json

import torch

from . import model as mm


def _time(fn, iters: int, warmup: int) -> float:
    """Average device time per launch: the `iters` launches are captured into
    one CUDA graph and replayed, so host launch cost is not measured."""
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(iters):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters * 1e3  # us


def gemv(args) -> dict:
    from . import ops

    tdt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[args.dtype]
    esz = 4 if args.dtype == "f32" else 2
    K, rows = args.k, args.rows
    g = torch.Generator(device="cuda").manual_seed(0)
    ws = [(torch.randn(rows, K, generator=g, device="cuda") * 0.02).to(tdt) for _ in range(args.copies)]
    x = torch.randn(K, generator=g, device="cuda")
    nw = torch.ones(K, device="cuda")
    if args.mode == "swiglu":
        out = torch.empty(rows // 2, device="cuda")
        fn = lambda i: ops.swiglu_matmul(out, x, nw, 1e-6, ws[i % len(ws)], rows // 2, K)
        extra = 2 * K * 4 + rows // 2 * 4
    elif args.mode == "norm":
        out = torch.empty(rows, device="cuda")
        fn = lambda i: ops.rmsnorm_matmul(out, x, nw, 1e-6, ws[i % len(ws)], rows, K)
        extra = 2 * K * 4 + rows * 4
    else:
        out = torch.zeros(rows, device="cuda")
        fn = lambda i: ops.matmul_residual(out, x, ws[i % len(ws)], rows, K)
        extra = K * 4 + 2 * rows * 4
    us = _time(fn, args.iters, args.warmup)
    algo = rows * K * esz + extra
    return {"op": f"gemv-{args.mode}", "rows": rows, "k": K, "dtype": args.dtype, "us": round(us, 2),
            "algo_bytes": algo, "gbs": round(algo / us / 1e3, 1)}


def attn(args) -> dict:
    from . import ops

    H, Hkv, D, ctx = args.hq, args.hkv, 128, args.ctx
    S = ctx + 16
    g = torch.Generator(device="cuda").manual_seed(0)
    kvt = torch.bfloat16 if args.kv == "bf16" else torch.float32
    kcs = [torch.randn(Hkv * S * D, generator=g, device="cuda").to(kvt) for _ in range(args.copies)]
    vcs = [torch.randn(Hkv * S * D, generator=g, device="cuda").to(kvt) for _ in range(args.copies)]
    qkv = torch.randn((H + 2 * Hkv) * D, generator=g, device="cuda")
    nw = torch.ones(D, device="cuda")
    rope = ops.rope_table(S, D, 1e6).cuda()
    split = args.split or ops.attn_default_split(Hkv, S)
    wsp = torch.zeros(ops.attn_workspace_bytes(H, Hkv, D, split) // 4 + 1, dtype=torch.int32, device="cuda")
    st = torch.tensor([0, ctx, 0, 0], dtype=torch.int32, device="cuda")
    out = torch.empty(H * D, device="cuda")
    fn = lambda i: ops.attn_decode(qkv, nw, nw, 1e-6, rope, kcs[i % len(kcs)], vcs[i % len(vcs)], S, st, out, H,
                                   Hkv, D, split, wsp)
    us = _time(fn, args.iters, args.warmup)
    algo = 2 * Hkv * (ctx + 1) * D * (2 if args.kv == "bf16" else 4) + (H + 2 * Hkv) * D * 4 + H * D * 4
    return {"op": "attn-decode", "kv": args.kv, "hq": H, "hkv": Hkv, "ctx": ctx, "split": split, "us": round(us, 2),
            "algo_bytes": algo, "gbs": round(algo / us / 1e3, 1)}


def gemm(args) -> dict:
    """The batched-prefill tcgen05 GEMM: M tokens x N outputs x K, bf16 hi/lo activations."""
    import ctypes as C

    from . import ops
    from ._lib import MF_PREFILL_RESID, MF_PREFILL_STORE, MF_PREFILL_SWIGLU, check, cuda_lib

    lib = cuda_lib()
    M, N, K = args.m, args.n, args.k
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn(M, K, generator=g, device="cuda")
    hi = a.to(torch.bfloat16)
    lo = (a - hi.float()).to(torch.bfloat16)
    ws = [(torch.randn(N, K, generator=g, device="cuda") * 0.02).to(torch.bfloat16) for _ in range(args.copies)]
    mode = {"store": MF_PREFILL_STORE, "resid": MF_PREFILL_RESID, "swiglu": MF_PREFILL_SWIGLU}[args.mode]
    y = torch.zeros(M, N, device="cuda") if mode != MF_PREFILL_SWIGLU else None
    hh = torch.empty(M, N // 2, dtype=torch.bfloat16, device="cuda") if mode == MF_PREFILL_SWIGLU else None
    hl = torch.empty_like(hh) if hh is not None else None
    P = lambda t: C.c_void_p(t.data_ptr()) if t is not None else None
    # the stream is looked up per launch: inside the graph capture it is torch's capture stream
    fn = lambda i: check(lib.mf_prefill_gemm(P(y), N if y is not None else 0, P(hi), P(lo), P(ws[i % len(ws)]), M, N,
                                             K, mode, P(hh), P(hl), C.c_void_p(ops._stream())))
    us = _time(fn, args.iters, args.warmup)
    flops = 2.0 * M * N * K  # algorithmic (the hi/lo split executes twice this on the tensor cores)
    return {"op": f"prefill-gemm-{args.mode}", "m": M, "n": N, "k": K, "us": round(us, 2),
            "tflops": round(flops / us / 1e6, 1), "tensor_tflops": round(2 * flops / us / 1e6, 1)}


def pattn(args) -> dict:
    """Batched-prefill causal attention of P tokens after pos0 cached positions:
    the tensor-core kernel (operand split included) or the SIMT kernel."""
    import ctypes as C

    from . import ops
    from ._lib import check, cuda_lib

    lib = cuda_lib()
    Pn, pos0, Hq, Hkv, D = args.p, args.pos0, args.hq, args.hkv, 128
    S = pos0 + Pn
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(Pn, Hq * D, generator=g, device="cuda")
    kc = torch.randn(Hkv, S, D, generator=g, device="cuda")
    vc = torch.randn(Hkv, S, D, generator=g, device="cuda")
    hi = torch.empty(Pn, Hq * D, dtype=torch.bfloat16, device="cuda")
    lo = torch.empty_like(hi)
    need = C.c_size_t()
    check(lib.mf_prefill_attention_scratch(Pn, S, Hq, Hkv, C.byref(need)))
    scratch = torch.empty(need.value, dtype=torch.uint8, device="cuda")
    P = lambda t: C.c_void_p(t.data_ptr())
    if args.kernel == "tc":
        fn = lambda i: check(lib.mf_prefill_attention_tc(P(hi), P(lo), P(q), P(kc), P(vc), S, Pn, pos0, Hq, Hkv, D,
                                                         P(scratch), need.value, 0, C.c_void_p(ops._stream())))
    else:
        fn = lambda i: check(lib.mf_prefill_attention(P(hi), P(lo), P(q), P(kc), P(vc), S, Pn, pos0, Hq, Hkv, D, 0,
                                                      C.c_void_p(ops._stream())))
    us = _time(fn, args.iters, args.warmup)
    st = C.c_int()
    check(lib.mf_prefill_status(C.byref(st), 1))
    # causal: token t attends to pos0 + t + 1 keys; 2 flops per multiply-add, QK^T and PV
    flops = 4.0 * Hq * D * (Pn * pos0 + Pn * (Pn + 1) / 2)
    return {"op": f"prefill-attn-{args.kernel}", "p": Pn, "pos0": pos0, "hq": Hq, "hkv": Hkv, "us": round(us, 2),
            "tflops": round(flops / us / 1e6, 1), "status": st.value}


def moe(args) -> dict:
    """One MoE layer's expert path at batch 1: router + top-k, grouped gate/up +
    SiLU over the k selected experts, grouped down + weighted residual. The
    expert weights of `--copies` layers rotate so each launch streams from HBM."""
    from . import ops

    E, k, F, d = args.experts, args.k_active, args.ff, args.d
    g = torch.Generator(device="cuda").manual_seed(0)
    wr = torch.randn(E, d, generator=g, device="cuda") * 0.02
    wgus = [(torch.randn(E * 2 * F, d, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
            for _ in range(args.copies)]
    wds = [(torch.randn(E * d, F, generator=g, device="cuda") * 0.02).to(torch.bfloat16) for _ in range(args.copies)]
    x = torch.randn(d, generator=g, device="cuda")
    nw = torch.ones(d, device="cuda")
    ids = torch.zeros(k, dtype=torch.int32, device="cuda")
    w = torch.zeros(k, device="cuda")
    scores = torch.zeros(E, device="cuda")
    h = torch.zeros(k * F, device="cuda")
    res = {}
    res["router_us"] = round(_time(lambda i: ops.router_topk(ids, w, scores, x, nw, 1e-6, wr, d, E, k), args.iters,
                                   args.warmup), 2)
    res["gate_up_us"] = round(_time(lambda i: ops.moe_swiglu(h, x, nw, 1e-6, wgus[i % len(wgus)], ids, k, F, d),
                                    args.iters, args.warmup), 2)
    res["down_us"] = round(_time(lambda i: ops.moe_down_residual(x, h, wds[i % len(wds)], ids, w, k, d, F),
                                 args.iters, args.warmup), 2)
    # the whole expert path as the model runs it: router + top-k, grouped gate/up, grouped down
    def layer(i):
        ops.router_topk(ids, w, scores, x, nw, 1e-6, wr, d, E, k)
        ops.moe_swiglu(h, x, nw, 1e-6, wgus[i % len(wgus)], ids, k, F, d)
        ops.moe_down_residual(x, h, wds[i % len(wds)], ids, w, k, d, F)

    res["layer_us"] = round(_time(layer, args.iters, args.warmup), 2)
    gu_bytes, dn_bytes = k * 2 * F * d * 2, k * d * F * 2
    res.update(op="moe-layer", experts=E, k=k, ff=F, d=d, gate_up_gbs=round(gu_bytes / res["gate_up_us"] / 1e3, 1),
               down_gbs=round(dn_bytes / res["down_us"] / 1e3, 1), router_bytes=E * d * 4,
               layer_gbs=round((gu_bytes + dn_bytes + E * d * 4) / res["layer_us"] / 1e3, 1))
    return res


def main():
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="what", required=True)
    a = sub.add_parser("gemv")
    a.add_argument("--rows", type=int, default=24576)
    a.add_argument("--k", type=int, default=4096)
    a.add_argument("--dtype", default="bf16")
    a.add_argument("--mode", default="swiglu", choices=["swiglu", "norm", "resid"])
    b = sub.add_parser("attn")
    b.add_argument("--hq", type=int, default=32)
    b.add_argument("--hkv", type=int, default=8)
    b.add_argument("--ctx", type=int, default=4096)
    b.add_argument("--split", type=int, default=0)
    b.add_argument("--kv", default="f32", choices=["f32", "bf16"], help="KV cache element type")
    c = sub.add_parser("gemm")
    c.add_argument("--m", type=int, default=4096)
    c.add_argument("--n", type=int, default=24576)
    c.add_argument("--k", type=int, default=4096)
    c.add_argument("--mode", default="swiglu", choices=["store", "resid", "swiglu"])
    f = sub.add_parser("pattn")
    f.add_argument("--p", type=int, default=4096)
    f.add_argument("--pos0", type=int, default=0)
    f.add_argument("--hq", type=int, default=32)
    f.add_argument("--hkv", type=int, default=8)
    f.add_argument("--kernel", default="tc", choices=["tc", "simt"])
    e = sub.add_parser("moe")
    e.add_argument("--experts", type=int, default=128)
    e.add_argument("--k-active", type=int, default=8)
    e.add_argument("--ff", type=int, default=768)
    e.add_argument("--d", type=int, default=2048)
    for p in (a, b, c, e, f):
        p.add_argument("--iters", type=int, default=20)
        p.add_argument("--warmup", type=int, default=5)
        p.add_argument("--copies", type=int, default=2)
    args = ap.parse_args()
    mm.init(1, [torch.cuda.current_device()])
    res = {"gemv": gemv, "attn": attn, "gemm": gemm, "moe": moe, "pattn": pattn}[args.what](args)
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
