#!/usr/bin/env python
"""Decode throughput of the Qwen3 token loop on B200 (batch 1).

Workload (default): the Qwen3-8B-shaped bf16 model (36 layers, hidden 4096,
32/8 heads, FFN 12288, untied lm_head, vocab 151936) as a seeded synthetic
GGUF; a 4096-token random prompt is prefilled, then greedy decode. One step is
one decode token at batch 1.

  value  tokens/s with everything resident in HBM: `steps` greedy tokens whose
         argmax feeds the next token on the device (chained CUDA-graph frames),
         timed with CUDA events on the launching stream.
  e2e    the same through the reference-facing C ABI call per token
         (mf_model_forward: step record H2D from pinned memory, frame, step
         record with the greedy id D2H), timed the same way.
Each step reads ~16.4 GB (weights + KV), far more than L2, so no flush is
needed between steps.

`--impl reference` runs the reference's own CPU token loop (oracle/_ref, built
from the reference sources; the oracle port if absent) on the host cores on a
bounded sample of the same workload.
Multi-GPU runs (torchrun, one rank per GPU) decode the same single stream
with tensor parallelism over the N GPUs (strong scaling): each rank holds a
1/N shard of every projection, the two all-reduces per layer are fused into
the GEMVs over NVLink peer memory. `value` is then the tokens/s of that one
stream, timed on the device as the max over ranks.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from minfer_b200.gguf_synth import CONFIGS, ensure_gguf, ensure_gguf_ranks  # noqa: E402

METRIC = "decode tokens/s (batch 1) and % HBM roofline at 1/2/4/8 B200; prefill tok/s"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return dict(PEAKS_FALLBACK), "fallback"


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def model_path(workload: str) -> Path:
    """Where the synthetic GGUF lives: $MF_MODEL_DIR, else /dev/shm when it has
    room for the file, else /tmp."""
    import shutil

    if os.environ.get("MF_MODEL_DIR"):
        d = Path(os.environ["MF_MODEL_DIR"])
        d.mkdir(parents=True, exist_ok=True)
        return d / f"minfer_b200_{workload}.gguf"
    need = CONFIGS[workload].weight_bytes() * 1.1 + (1 << 30)
    for d in ("/dev/shm", "/tmp"):
        p = Path(d) / f"minfer_b200_{workload}.gguf"
        if p.exists():
            return p
        if Path(d).is_dir() and shutil.disk_usage(d).free > need:
            return p
    return Path("/tmp") / f"minfer_b200_{workload}.gguf"


def prepare_model(workload: str, rank: int, world: int):
    """The workload's synthetic GGUF (written once; with several ranks every
    rank draws a share of the weights)."""
    path = model_path(workload)
    cfg = CONFIGS[workload]
    if world > 1:
        import torch.distributed as dist

        ensure_gguf_ranks(path, cfg, rank, world, dist.barrier)
    else:
        ensure_gguf(path, cfg)
    return str(path), cfg


class Clocks:
    """nvidia-smi sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.tmp,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        self.tmp.flush()
        rows = [r.split(",") for r in Path(self.tmp.name).read_text().strip().splitlines() if r.strip()]
        os.unlink(self.tmp.name)
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def token_bytes(info, ctx: int) -> float:
    """Algorithmic bytes of one decode token at context ctx: every weight byte
    the forward reads (lm_head included) plus the KV rows read (ctx+1 rows)."""
    return float(info.read_bytes_logits) + float(info.kv_bytes_per_pos) * (ctx + 1)


def time_dominant_kernel(cfg, peaks, iters: int = 20) -> dict:
    """The fused gate/up + SiLU GEMV of one layer (the largest weight stream of
    a dense decode step), timed alone with CUDA events on torch's stream."""
    import torch

    from minfer_b200 import ops

    d, F = cfg.d_model, cfg.d_ff
    g = torch.Generator(device="cuda").manual_seed(1)
    w = (torch.randn(2 * F, d, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    x = torch.randn(d, generator=g, device="cuda")
    nw = torch.ones(d, device="cuda")
    h = torch.empty(F, device="cuda")
    for _ in range(3):
        ops.swiglu_matmul(h, x, nw, 1e-6, w, F, d)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        ops.swiglu_matmul(h, x, nw, 1e-6, w, F, d)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / iters
    algo = 2 * F * d * 2 + 2 * d * 4 + F * 4
    achieved = algo / (ms * 1e-3) / 1e9
    traffic = None
    prof = ROOT / "profiles" / "gemv_swiglu_qwen3-8b.txt"
    if prof.exists():
        for line in prof.read_text().splitlines():
            if line.strip().startswith("dram_bytes_per_launch:"):
                traffic = float(line.split(":")[1])
    return {"kernel": "gemv_tma_kernel<W_BF16, 8, 2, X_NORM, Y_SWIGLU> (RMSNorm + gate/up + SiLU over a "
                      "TMA bulk-copy ring, one layer)",
            "bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": traffic, "algo_bytes": algo,
            "avg_launch_us": round(ms * 1e3, 2)}


def prefill_line(cfg, ctx: int, seconds: float, batched: bool, peaks, world: int = 1) -> dict:
    """Prefill tok/s and its tensor roofline. Algorithmic FLOPs of the prompt:
    2 x linear params each token uses x tokens (Q/K/V/O, gate/up/down per
    layer: for MoE the router and the k selected experts; the lm_head runs
    once) + causal attention 4 x L x Hq x D x (sum of context lengths). The
    hi/lo operand split executes the linear part twice."""
    L, d, Hq, Hkv, D, F = cfg.n_layers, cfg.d_model, cfg.n_heads, cfg.n_kv_heads, cfg.d_head, cfg.d_ff
    ffn = 3 * d * F * (cfg.n_active if cfg.n_experts else 1) + (d * cfg.n_experts if cfg.n_experts else 0)
    lin = 2.0 * L * (d * (Hq + 2 * Hkv) * D + Hq * D * d + ffn) * ctx
    att = 4.0 * L * Hq * D * (ctx * (ctx + 1) / 2)
    out = {"tokens": ctx, "seconds": round(seconds, 4), "tok_per_s": round(ctx / seconds, 1),
           "method": ("batched: tcgen05 GEMMs on fp32 activations split into bf16 hi+lo, tcgen05 causal attention"
                      + ("; MoE: fp32 router, tokens grouped by expert, grouped expert GEMMs" if cfg.n_experts
                         else "")
                      + (f", tensor-parallel over {world} GPUs (partials exchanged per projection)" if world > 1
                         else "") if batched else "token-by-token decode frames")}
    if batched:
        achieved = (lin + att) / seconds / 1e12
        peak = peaks["bf16_tflops"] * world  # aggregate over the GPUs
        out["roofline"] = {"bound": "tensor", "algo_tflop": round((lin + att) / 1e12, 2),
                           "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TFLOP/s",
                           "frac": round(achieved / peak, 4),
                           "note": "algorithmic FLOPs; the hi/lo split runs the linear part twice on the tensor cores"}
    return out


def run_reference_cpu(path: str, ctx: int, steps: int, warmup: int, threads: int) -> dict:
    """Reference CPU token loop at context ctx: `steps` timed decode forwards."""
    from oracle import oracle_py

    with tempfile.TemporaryDirectory() as td:
        arch = oracle_py.ref_binary()[1]
        if oracle_py.ref_available():
            res = oracle_py.run_reference(path, f"{td}/r", bench_context=ctx, bench_steps=steps,
                                          bench_warmup=warmup, threads=threads, timeout=1800)
            kind = "reference"
        else:
            pm = oracle_py.PortModel(path, max_seq=ctx + steps + warmup + 1)
            ts = []
            for s in range(warmup + steps):
                t0 = time.perf_counter()
                pm.forward(1 + s, ctx + s, True)
                if s >= warmup:
                    ts.append(time.perf_counter() - t0)
            res = {"tok_per_s": len(ts) / sum(ts), "seconds": sum(ts)}
            kind = "port"
            arch = "-march=x86-64-v3 (oracle restatement)"
    return {"value": res["tok_per_s"], "unit": "tokens/s", "cores": threads, "kind": kind,
            "sample": f"{steps} decode tokens (+{warmup} warm-up) at context {ctx} on the same GGUF, "
                      f"KV rows below the context zero-filled, OMP_NUM_THREADS={threads}",
            "seconds": res["seconds"], "omp_num_threads": threads, "host": host_cpu(),
            "build": f"g++ 13 -O3 {arch} -fopenmp; the reference's NEON GEMVs as 128-bit FMA/F16C/SSE ops"}


PARITY_PROMPT = 64  # prompt tokens of the multi-GPU parity check
PARITY_GEN = 16  # greedy ids compared
MARGIN_TOL = 1e-4  # a step whose top-2 logit gap (single-GPU side) is below this may flip


def tp_parity(m, path: str, prompt, info, rank: int, world: int, local_rank: int) -> dict:
    """Greedy ids of the sharded model against a single-GPU run of the whole
    model on rank 0's GPU, for the first PARITY_PROMPT prompt ids. Rank 0
    decodes free-running (ids and top-2 logit margins); every rank then
    decodes teacher-forced on those ids. An id may differ only where the
    single-GPU margin is below MARGIN_TOL, and every rank must produce the
    same ids. Runs after the timed regions (it rewrites the KV cache)."""
    import torch.distributed as dist

    from minfer_b200 import model as mm

    p = prompt[:PARITY_PROMPT]
    ref = [None, None]
    if rank == 0:
        single = mm.Qwen3Model(path, mm.RunParams(num_iters=PARITY_GEN, max_seq_len=len(p) + PARITY_GEN + 1),
                               device=local_rank).set_device("cuda")
        ids, mg, _ = single.generate(p, PARITY_GEN, margins=True)
        ref = [[int(v) for v in ids], [float(v) for v in mg]]
        single.close()
        del single
    box = [ref]
    dist.broadcast_object_list(box, src=0)
    ref_ids, ref_mg = box[0]
    ids, _, _ = m.generate(p, PARITY_GEN, forced=np.array(ref_ids, np.uint32))
    ids = [int(v) for v in ids]
    every = [None] * world
    dist.all_gather_object(every, ids)
    same = all(e == every[0] for e in every)
    events = [i for i, (a, b) in enumerate(zip(ids, ref_ids)) if a != b]
    bad = [i for i in events if ref_mg[i] >= MARGIN_TOL]
    return {"ok": same and not bad, "ids_same_on_all_ranks": same, "compared": len(ref_ids),
            "prompt_tokens": len(p), "tolerance_events": events, "mismatches": bad,
            "min_margin": round(min(ref_mg), 6) if ref_mg else None,
            "ids": ids, "against": "single-GPU decode of the whole model (teacher-forced, margin rule)"}


def llama_bench_record(m, batched: bool) -> dict:
    """BaseModel::benchmark's numbers (pp512 then tg128 of random ids, each
    tg step one host-driven frame) from this runtime."""
    st = m.benchmark(token_prefill=not batched)
    return {"pp512_seconds": round(st.prefill_time, 4), "tg128_tok_per_s": round(st.throughput, 2),
            "bandwidth_gbs": round(st.bandwidth, 1),
            "prefill": "batched tensor-core prefill" if batched else "token by token, as the reference",
            "note": "the reference's formula: bytes it counts (lm_head every step) / (pp + tg time)"}


def llama_bench_main(args) -> None:
    """The reference's own published loop (README tg128 rows) on one model:
    this runtime (batched and token-by-token pp512) next to the reference's
    CPU build running BaseModel::benchmark unchanged. Seed 30, 4096-token cache."""
    import torch

    from minfer_b200 import model as mm
    from oracle import oracle_py

    torch.cuda.set_device(0)
    mm.init(1, [0])
    path, cfg = prepare_model(args.workload, 0, 1)
    rp = mm.RunParams(num_iters=128, max_seq_len=4096, seed=30)
    m = mm.Qwen3Model(path, rp).set_device("cuda")
    ours = llama_bench_record(m, True)
    ours_tok = llama_bench_record(m, False)
    line = {"metric": "tg128 tokens/s (BaseModel::benchmark: pp512 + tg128, seed 30)", "workload": args.workload,
            "unit": "tokens/s", "value": ours["tg128_tok_per_s"], "minfer_b200": ours,
            "minfer_b200_token_prefill": ours_tok}
    if oracle_py.ref_available():
        thr = host_threads()
        with tempfile.TemporaryDirectory() as td:
            r = oracle_py.run_reference(path, f"{td}/r", llama_bench=True, seed=30, max_seq=4096, threads=thr,
                                        timeout=1800)
        line["reference_cpu"] = {"pp512_seconds": round(r["prefill_time"], 3),
                                 "tg128_tok_per_s": round(r["throughput"], 3), "bandwidth_gbs": round(r["bandwidth"], 2),
                                 "omp_num_threads": thr, "build": oracle_py.ref_binary()[1]}
    print(json.dumps(line), flush=True)


def measure_long_context(workload: str, ctx: int, steps: int, warmup: int, rank: int, world: int, local_rank: int,
                         peaks: dict, kv_dtype: str = "f32", parity: bool = False) -> dict:
    """Decode of a second workload, the same way as the main line (prefill of
    a random prompt: batched on the tensor cores when the model allows it,
    else token by token; chained greedy decode timed with CUDA events, max
    over ranks): tokens/s and the HBM roofline fraction per GPU, prefill
    tokens/s, exchange status. kv_dtype "bf16" runs it with the opt-in bf16
    KV cache (the reference's cache is fp32). parity (N > 1): the sharded
    model's greedy ids against a single-GPU decode on rank 0 (margin rule)."""
    import torch

    from minfer_b200 import model as mm
    from minfer_b200 import tp
    from minfer_b200._lib import check, cuda_lib

    lib = cuda_lib()
    t0 = time.perf_counter()
    path, cfg = prepare_model(workload, rank, world)
    t_gen = time.perf_counter() - t0
    n_tok = warmup + steps + 4
    t0 = time.perf_counter()
    m = mm.Qwen3Model(path, mm.RunParams(num_iters=n_tok, max_seq_len=ctx + n_tok + 2), device=local_rank,
                      tp_rank=rank, tp_size=world, kv_dtype=kv_dtype)
    m.set_device("cuda")
    tp.connect(m)
    t_load = time.perf_counter() - t0
    info = m.info
    prompt = mm.random_prompt(ctx, info.vocab_size, 30)
    ms = C.c_float()
    check(lib.mf_timer_start(0))
    batched = m.prefill(prompt, 0, True, False)
    if not batched:
        for i, t in enumerate(prompt):
            m.forward(int(t), i, i == ctx - 1, False)
    check(lib.mf_timer_stop(0, C.byref(ms)))
    prefill_s = ms.value / 1e3
    tok = m.argmax()
    tok = m.decode_chained(tok, ctx, warmup)

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        import torch.distributed as dist

        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()
    check(lib.mf_timer_start(0))
    m.decode_chained(tok, ctx + warmup, steps)
    check(lib.mf_timer_stop(0, C.byref(ms)))
    dev_ms = max_over_ranks(ms.value)
    prefill_s = max_over_ranks(prefill_s)
    tb = token_bytes(info, ctx + warmup + steps // 2)
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([tb], device="cuda", dtype=torch.float64)
        dist.all_reduce(t)
        tb = t.item()
    status = int(max_over_ranks(float(m.comm_status())))
    par = tp_parity(m, path, prompt, info, rank, world, local_rank) if parity and world > 1 else None
    m.close()
    step_gbs = tb / (dev_ms / steps / 1e3) / 1e9 / world
    return {"workload": f"{workload} greedy decode at batch 1 after a {ctx}-token prompt", "context": ctx,
            "kv_dtype": kv_dtype, "tok_per_s": round(steps / (dev_ms / 1e3), 2), "ms_per_step": round(dev_ms / steps, 3), "steps": steps,
            "bytes_per_token": tb, "hbm_roofline": {"achieved_gbs_per_gpu": round(step_gbs, 1),
                                                    "peak_gbs": peaks["hbm_gbs"],
                                                    "frac": round(step_gbs / peaks["hbm_gbs"], 4)},
            "prefill_tok_per_s": round(ctx / prefill_s, 1),
            "prefill": "batched (tensor cores)" if batched else "token by token",
            **({"parity_ok": par["ok"], "parity": par} if par else {}), "exchange_status": status,
            "parallelism": "single" if world == 1 else (f"ep{world}" if info.expert_parallel else f"tp{world}"),
            "load_seconds": round(t_load, 1),
            "file_seconds": round(t_gen, 1)}


def guarded(fn, *args, **kw) -> dict:
    """A secondary record: a failure is reported in the record instead of
    ending the run (the main line is already measured)."""
    try:
        return fn(*args, **kw)
    except Exception as e:  # reported, not fatal
        import gc

        gc.collect()  # (drops the failed record's model, whose frames the exception held)
        return {"error": f"{type(e).__name__}: {str(e)[:300]}"}


def measure_sampled(workload: str, ctx: int, gen: int, local_rank: int) -> dict:
    """Sampled decode through the public generate call (the 1.7B workload's
    sampler: top-k 20, temperature 0.7, top-p 0.9, seed 42) after a ctx-token
    prompt: tokens/s of the decode loop with the draws on the device (chained
    frames) and with the host loop (MF_DEVICE_SAMPLE=0); both must give the
    same ids."""
    from minfer_b200 import model as mm

    path, _ = prepare_model(workload, 0, 1)
    rp = mm.RunParams(num_iters=gen, max_seq_len=ctx + gen + 2, top_k=20, temp=0.7, top_p=0.9, seed=42)
    out = {"workload": f"{workload}, {ctx}-token prompt, {gen} sampled tokens (top-k 20, T 0.7, top-p 0.9)"}
    ids = {}
    for mode in ("device", "host"):
        if mode == "host":
            os.environ["MF_DEVICE_SAMPLE"] = "0"
        try:
            m = mm.Qwen3Model(path, rp, device=local_rank).set_device("cuda")
            prompt = mm.random_prompt(ctx, m.info.vocab_size, 42)
            m.generate(prompt[:64], 8)  # warm-up (graphs captured)
            got, _, st = m.generate(prompt, gen)
            ids[mode] = [int(v) for v in got]
            out[f"{mode}_tok_per_s"] = round(st.throughput, 1)
            m.close()
        finally:
            os.environ.pop("MF_DEVICE_SAMPLE", None)
    out["same_ids"] = ids["device"] == ids["host"]
    return out


def host_cpu() -> dict:
    """The host's CPU as lscpu reports it (model, sockets, physical cores,
    logical CPUs), the CPUs this process may run on, the cgroup CPU quota and
    the RAM. `threads` = physical cores, capped by the CPUs the process may use
    (more OpenMP threads than usable CPUs only time-slice)."""
    info = {"model": None, "sockets": None, "cores_per_socket": None, "threads_per_core": None, "logical": None}
    try:
        out = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
        keys = {"Model name": "model", "Socket(s)": "sockets", "Core(s) per socket": "cores_per_socket",
                "Thread(s) per core": "threads_per_core", "CPU(s)": "logical"}
        for line in out.splitlines():
            k, _, v = line.partition(":")
            if k.strip() in keys and info[keys[k.strip()]] is None:
                v = v.strip()
                info[keys[k.strip()]] = int(v) if v.isdigit() else v
    except (OSError, subprocess.SubprocessError):
        pass
    phys = None
    if isinstance(info["sockets"], int) and isinstance(info["cores_per_socket"], int):
        phys = info["sockets"] * info["cores_per_socket"]
    info["physical_cores"] = phys
    try:
        usable = len(os.sched_getaffinity(0))
    except AttributeError:
        usable = os.cpu_count() or 1
    info["usable_cpus"] = usable
    quota = None
    try:
        q, per = Path("/sys/fs/cgroup/cpu.max").read_text().split()
        if q != "max":
            quota = round(int(q) / int(per), 2)
    except (OSError, ValueError):
        pass
    info["cgroup_cpu_quota"] = quota
    try:
        info["ram_gb"] = round(os.sysconf("SC_PAGE_SIZE") * os.sysconf("SC_PHYS_PAGES") / 1e9, 1)
    except (ValueError, OSError):
        info["ram_gb"] = None
    t = phys or usable
    t = min(t, usable)
    if quota:
        t = min(t, max(1, int(quota)))
    info["threads"] = max(1, t)
    return info


def host_threads() -> int:
    return host_cpu()["threads"]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="minfer_b200", choices=["minfer_b200", "reference"])
    ap.add_argument("--workload", default="qwen3-8b-bf16", choices=sorted(CONFIGS))
    ap.add_argument("--context", type=int, default=4096, help="prompt tokens prefilled before decode")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-steps", type=int, default=16)
    ap.add_argument("--long-workload", default="qwen3-32b-bf16", choices=sorted(CONFIGS),
                    help="second record: this model decoded after a long prompt (the scaling target)")
    ap.add_argument("--long-context", type=int, default=32768)
    ap.add_argument("--no-long", action="store_true", help="skip the long-context record")
    ap.add_argument("--no-long-kv-bf16", action="store_true",
                    help="skip the long-context run with the opt-in bf16 KV cache")
    ap.add_argument("--moe-workload", default="qwen3-30b-a3b-bf16", choices=sorted(CONFIGS))
    ap.add_argument("--moe-context", type=int, default=1024)
    ap.add_argument("--no-moe", action="store_true", help="skip the MoE record")
    ap.add_argument("--no-sampled", action="store_true", help="skip the sampled-decode record")
    ap.add_argument("--llama-bench", action="store_true",
                    help="only the reference's benchmark loop (pp512 + tg128, seed 30) on --workload, this runtime "
                         "and the reference CPU build side by side (one GPU)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank, world, local_rank = dist_env()
    cfgshape = CONFIGS[args.workload]
    config = {"workload": f"{args.workload} greedy decode at batch 1 after a {args.context}-token prompt",
              "context": args.context, "batch": 1,
              "l2": "inputs larger than L2 (each step streams all weights and the KV cache)",
              "parallelism": "single" if world == 1 else
              (f"ep{world}" if cfgshape.n_experts > 0 and (cfgshape.n_kv_heads % world or
                                                          os.environ.get("MF_MOE_EP") == "1") else f"tp{world}")}

    if args.llama_bench:
        llama_bench_main(args)
        return

    if args.impl == "reference":
        if rank != 0:
            return
        path, _ = prepare_model(args.workload, 0, 1)
        thr = host_threads()
        cb = run_reference_cpu(path, args.context, args.steps, args.warmup, thr)
        line = {"metric": METRIC, "value": round(cb["value"], 4), "unit": "tokens/s", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 / cb["value"], 3),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": config, "impl": "reference", "cpu_baseline": cb,
                "e2e": {"value": round(cb["value"], 4), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch

    torch.cuda.set_device(local_rank)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))
    from minfer_b200 import model as mm
    from minfer_b200 import tp
    from minfer_b200._lib import check, cuda_lib

    mm.init(1, [local_rank])
    lib = cuda_lib()
    path, cfg = prepare_model(args.workload, rank, world)
    ctx = args.context
    n_tok = args.warmup + 2 * args.steps + 4
    t_load = time.perf_counter()
    m = mm.Qwen3Model(path, mm.RunParams(num_iters=n_tok, max_seq_len=ctx + n_tok + 2), device=local_rank,
                      tp_rank=rank, tp_size=world)
    m.set_device("cuda")
    tp.connect(m)
    t_load = time.perf_counter() - t_load
    info = m.info
    prompt = mm.random_prompt(ctx, info.vocab_size, 30)

    # prefill: batched on the tensor cores (tcgen05 GEMMs) when the model
    # allows it, else token by token through the decode frames; timed on the device
    ms = C.c_float()
    check(lib.mf_timer_start(0))
    batched = m.prefill(prompt, 0, True, False)
    if not batched:
        for i, t in enumerate(prompt):
            m.forward(int(t), i, i == ctx - 1, False)
    check(lib.mf_timer_stop(0, C.byref(ms)))
    prefill_s = ms.value / 1e3
    tok = m.argmax()
    if batched:
        # once more, warm (the first pass includes one-time set-up: buffers, graphs)
        check(lib.mf_timer_start(0))
        m.prefill(prompt, 0, True, False)
        check(lib.mf_timer_stop(0, C.byref(ms)))
        prefill_s = min(prefill_s, ms.value / 1e3)
        tok = m.argmax()

    # warm-up (graphs captured, clocks up)
    tok = m.decode_chained(tok, ctx, args.warmup)
    pos = ctx + args.warmup

    def barrier():
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        import torch.distributed as dist

        t = torch.tensor([v], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    # ---- value: chained device-side decode
    barrier()
    with Clocks(local_rank) as clk:
        check(lib.mf_timer_start(0))
        tok = m.decode_chained(tok, pos, args.steps)
        check(lib.mf_timer_stop(0, C.byref(ms)))
    barrier()
    dev_ms = max_over_ranks(ms.value)
    pos += args.steps
    value = args.steps / (dev_ms / 1e3)

    # ---- e2e: one reference-facing call per token, host in the loop
    barrier()
    check(lib.mf_timer_start(0))
    for i in range(args.steps):
        m.forward(int(tok), pos + i, True, False)
        tok = m.argmax()
    check(lib.mf_timer_stop(0, C.byref(ms)))
    barrier()
    e2e_ms = max_over_ranks(ms.value)
    e2e = args.steps / (e2e_ms / 1e3)

    # ---- multi-GPU correctness: the sharded decode vs a single-GPU decode of
    # the same prompt (margin rule), then every rank's exchange status
    status = m.comm_status()
    parity = tp_parity(m, path, prompt, info, rank, world, local_rank) if world > 1 else None

    peaks, peak_kind = load_peaks()
    prefill_max_s = max_over_ranks(prefill_s)
    ctx_mid = ctx + args.warmup + args.steps // 2
    # bytes every rank reads per token, summed over ranks (the replicated
    # norms and embedding row are a few KB per layer)
    tb = token_bytes(info, ctx_mid)
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([tb], device="cuda", dtype=torch.float64)
        dist.all_reduce(t)
        tb = t.item()
    step_gbs = tb / (dev_ms / args.steps / 1e3) / 1e9 / world  # per GPU
    status = max(status, m.comm_status())
    # the reference's benchmark loop (pp512 + tg128) on the same model (N=1)
    # (the reference's pp512 + tg128 loop needs a cache of at least 512 positions)
    lb = llama_bench_record(m, batched) if world == 1 and ctx + n_tok + 2 >= 512 else None
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([status], device="cuda", dtype=torch.int32)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        status = int(t.item())
    roof = time_dominant_kernel(cfgshape, peaks) if rank == 0 else None

    # ---- the long-context record (the 32B-shaped model after a 32K prompt by default)
    long_rec = None
    if not args.no_long:
        import shutil

        lp = model_path(args.long_workload)
        room = lp.exists() or shutil.disk_usage(lp.parent).free > CONFIGS[args.long_workload].weight_bytes() * 1.05
        if world > 1:
            import torch.distributed as dist

            box = [room]
            dist.broadcast_object_list(box, src=0)  # every rank takes the same branch
            room = box[0]
        if room:
            m.close()
            long_rec = guarded(measure_long_context, args.long_workload, args.long_context, args.steps,
                               args.warmup, rank, world, local_rank, peaks)
            if not args.no_long_kv_bf16 and "error" not in long_rec:  # the same run with the opt-in bf16 KV cache
                long_rec["kv_bf16"] = guarded(measure_long_context, args.long_workload, args.long_context, args.steps,
                                              args.warmup, rank, world, local_rank, peaks, "bf16")
        else:
            long_rec = {"skipped": f"no room for the {args.long_workload} file under {lp.parent}"}

    # ---- the MoE record (the 30B-A3B shape; expert parallelism at N > 1)
    moe_rec = None
    if not args.no_moe and args.moe_workload != args.workload:
        import shutil

        mp = model_path(args.moe_workload)
        room = mp.exists() or shutil.disk_usage(mp.parent).free > CONFIGS[args.moe_workload].weight_bytes() * 1.05
        if world > 1:
            import torch.distributed as dist

            box = [room]
            dist.broadcast_object_list(box, src=0)
            room = box[0]
        if room:
            moe_rec = guarded(measure_long_context, args.moe_workload, args.moe_context, args.steps, args.warmup,
                              rank, world, local_rank, peaks, parity=True)
        else:
            moe_rec = {"skipped": f"no room for the {args.moe_workload} file under {mp.parent}"}

    sampled = None
    if world == 1 and not args.no_sampled:
        try:
            sampled = measure_sampled("qwen3-1.7b-bf16", 512, 256, local_rank)
        except Exception as e:  # reported, not fatal
            sampled = {"error": str(e)[:200]}

    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and world == 1:  # rank 0 at N=1 only (other ranks would compete for cores)
            try:
                cpu = run_reference_cpu(path, ctx, args.cpu_steps, 1, host_threads())
            except Exception as e:  # reported, not fatal
                cpu = {"value": None, "error": str(e)[:200]}
        # embed + lm_head, and per layer QKV, attention, O, gate/up, down (+ router GEMV and top-k for MoE)
        launches_per_step = 2 + 5 * info.n_layers if info.n_experts == 0 else 2 + 7 * info.n_layers
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "compute": "fp32 accumulate, fp32 activations/KV",
            "data": "synthetic (seeded GGUF, random prompt ids)", "config": config,
            "e2e": {"value": round(e2e, 3), "unit": "tokens/s", "h2d_bytes_per_step": 16, "d2h_bytes_per_step": 16,
                    "ms_per_step": round(e2e_ms / args.steps, 4)},
            "gpu_launches": launches_per_step * args.steps,
            "hbm_roofline": {"bytes_per_token": tb, "achieved_gbs": round(step_gbs, 1), "peak_gbs": peaks["hbm_gbs"],
                             "frac": round(step_gbs / peaks["hbm_gbs"], 4), "peak_kind": peak_kind},
            "roofline": dict(roof, peak_kind=peak_kind),
            "prefill": prefill_line(cfgshape, ctx, prefill_max_s, batched, peaks, world),
            "cpu_baseline": cpu, "clocks": clk.summary(), "load_seconds": round(t_load, 2),
        }
        if lb:
            line["llama_bench"] = lb
        if long_rec:
            line["long_context"] = long_rec
        if moe_rec:
            line["moe"] = moe_rec
        if sampled:
            line["sampled"] = sampled
        if world > 1:
            line["tp"] = {"size": world, "exchange_status": status,
                          "note": "hbm_roofline.achieved_gbs is per GPU; bytes_per_token summed over ranks"}
            line["parity_ok"] = bool(parity["ok"]) and status == 0
            line["exchange_status"] = status
            line["parity"] = parity
        print(json.dumps(line), flush=True)
    moe_bad = bool(moe_rec) and (moe_rec.get("parity_ok") is False or moe_rec.get("exchange_status", 0) != 0 or
                                 "error" in moe_rec)
    failed = world > 1 and (not (parity["ok"] and status == 0) or moe_bad)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    if failed:
        sys.exit(3)


if __name__ == "__main__":
    main()
