"""One rank of the tensor-parallel parity run (launched by test_gpu_tp.py under
torch.distributed.run, one process per GPU).

Per model, every rank loads its shard, connects over CUDA IPC and checks:
  * the stand-alone all-reduce is exact (rank-order fp32 sum);
  * greedy ids under teacher forcing vs the oracle (margin rule), margins
    (logit top-2 gaps) within the logits tolerance, step-0 logits within it;
  * free-running greedy ids equal the oracle's up to the first tolerance
    event and are identical on every rank;
  * sampled ids (temperature 0.7, top-k 20, top-p 0.9, seed 42) identical on
    every rank and equal to the oracle's unless the flip rule
    (tests/sampling_rule.py) explains a flip by the logits' error;
  * the chained (device-fed) decode ends on the host loop's last id;
  * no exchange wait gave up.
Exits non-zero on the first failure.
"""
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

from conftest import TINY, tiny_model  # noqa: E402
from minfer_b200 import model as mm  # noqa: E402
from minfer_b200 import ops  # noqa: E402
from minfer_b200._lib import MF_COMM_HANDLE_BYTES, check, cuda_lib  # noqa: E402
from minfer_b200.tp import connect, env_ranks, gather_handles  # noqa: E402
from oracle.oracle_py import PortModel, uniform_draws  # noqa: E402
from sampling_rule import check_sampled  # noqa: E402
from test_gpu_model import oracle_sampled  # noqa: E402

MARGIN_TOL = 1e-4


def logit_tol(dtype):
    return 1e-3 if dtype == "f32" else 2e-2


def same_on_all_ranks(arr) -> bool:
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, [int(v) for v in arr])
    return all(o == out[0] for o in out)


def check_allreduce(rank, world, device):
    import ctypes as C

    lib = cuda_lib()
    comm = C.c_void_p()
    n = 5120
    check(lib.mf_comm_create(0, rank, world, n, 0, C.byref(comm)))
    h = (C.c_char * MF_COMM_HANDLE_BYTES)()
    check(lib.mf_comm_handle(comm, h, MF_COMM_HANDLE_BYTES))
    blob = b"".join(gather_handles(bytes(h)))
    check(lib.mf_comm_connect(comm, C.create_string_buffer(blob, len(blob)), len(blob)))
    dist.barrier()
    rng = np.random.default_rng(1000 + rank)
    res = np.random.default_rng(7).standard_normal(n).astype(np.float32)  # same residual on every rank
    st = torch.zeros(8, dtype=torch.int32, device=device)  # step record; frame field tags the messages
    for it in range(6):
        st[4] = 1 + it // 2  # two exchanges (seq 0, 1) per frame
        part = rng.standard_normal(n).astype(np.float32)
        parts = [None] * world
        dist.all_gather_object(parts, part)
        exp = res.copy()
        for p in parts:
            exp = exp + p  # rank order, fp32
        xo = torch.empty(n, device=device)
        pt = torch.from_numpy(part).to(device)
        rt = torch.from_numpy(res).to(device)
        check(lib.mf_allreduce(C.c_void_p(xo.data_ptr()), C.c_void_p(rt.data_ptr()), C.c_void_p(pt.data_ptr()), n,
                               comm, it % 2, C.c_void_p(st.data_ptr()), C.c_void_p(ops._stream())))
        got = xo.cpu().numpy()
        assert np.array_equal(got, exp), f"all-reduce mismatch at call {it}: {np.abs(got - exp).max()}"
    st = C.c_int()
    check(lib.mf_comm_status(comm, C.byref(st), 1))
    assert st.value == 0, f"exchange status {st.value}"
    dist.barrier()
    lib.mf_comm_destroy(comm)


def check_model(name, rank, world):
    cfg = TINY[name]
    path = tiny_model(name)
    P, G = 12, 32
    prompt = mm.random_prompt(P, cfg.vocab, 30)
    orc = PortModel(path, max_seq=P + G + 1)
    ref_ids, ref_mg = orc.generate(prompt, G)

    def load(**kw):
        m = mm.Qwen3Model(path, mm.RunParams(num_iters=G, max_seq_len=P + G + 2, **kw), tp_rank=rank,
                          tp_size=world).set_device("cuda")
        connect(m)
        return m

    m = load()
    assert m.info.tp_size == world and m.info.tp_rank == rank
    # step-0 logits (full vocabulary gathered on every rank)
    orc0 = PortModel(path, max_seq=P + 1)
    for i, t in enumerate(prompt):
        orc0.forward(int(t), i, i == P - 1)
        m.forward(int(t), i, i == P - 1, i == P - 1)
    err = np.max(np.abs(orc0.logits() - m.logits()))
    assert err <= logit_tol(cfg.dtype), f"{name}: step-0 logits max-abs {err}"
    ref_e = None
    if cfg.n_experts > 0:
        # the router runs on every rank: every rank's expert ids per layer match the oracle's
        orc_e = PortModel(path, max_seq=P + 1)
        orc_e.record_experts(True)
        me = load()
        for i, t in enumerate(prompt):
            orc_e.forward(int(t), i, True)
            me.forward(int(t), i, True, False)
            ref_e, _ = orc_e.recorded_experts(cfg.n_active)
            for layer in range(cfg.n_layers):
                ids, _ = me.experts(layer)
                assert list(ids) == list(ref_e[i * cfg.n_layers + layer]), f"{name}: experts differ at {i}/{layer}"
        assert me.comm_status() == 0
        me.close()
    assert m.argmax() == int(np.argmax(m.logits()))
    if cfg.dtype == "bf16":
        # batched prefill on the tensor cores, partials exchanged per projection
        # (dense) or per layer's experts (MoE, expert parallelism); one pass, and
        # 5-row chunks: alternating slots and cached history
        for chunk in (None, "5"):
            if chunk:
                os.environ["MF_PREFILL_CHUNK"] = chunk
            mp = load()
            assert mp.prefill(prompt, 0, True, True), f"{name}: batched prefill not taken"
            err = np.max(np.abs(orc0.logits() - mp.logits()))
            assert err <= logit_tol(cfg.dtype), f"{name}: batched-prefill logits max-abs {err} (chunk {chunk})"
            assert mp.argmax() == int(np.argmax(mp.logits()))
            assert same_on_all_ranks([mp.argmax()]), f"{name}: ranks disagree after batched prefill"
            if ref_e is not None:  # every rank routed the prompt like the oracle
                n_last = P if not chunk else P - (P - 1) // int(chunk) * int(chunk)
                want = ref_e.reshape(P, cfg.n_layers, cfg.n_active)[P - n_last:]
                for layer in range(cfg.n_layers):
                    got, _ = mp.prefill_experts(layer, n_last)
                    assert np.array_equal(got, want[:, layer]), f"{name}: prefill experts differ at layer {layer}"
            assert mp.comm_status() == 0
            mp.close()
            os.environ.pop("MF_PREFILL_CHUNK", None)
    # teacher-forced greedy
    ids, mg, st = m.generate(prompt, G, forced=ref_ids, margins=True)
    events = [i for i in range(G) if ids[i] != ref_ids[i]]
    for i in events:
        assert ref_mg[i] < MARGIN_TOL, f"{name}: id mismatch at step {i}, margin {ref_mg[i]}"
    np.testing.assert_allclose(mg, ref_mg, atol=logit_tol(cfg.dtype))
    assert len(events) <= 1 and st.num_tokens_gen == G
    # free-running greedy
    m2 = load()
    free, _, _ = m2.generate(prompt, G)
    first = events[0] if events else G
    assert list(free[:first]) == list(ref_ids[:first]), f"{name}: free-running greedy diverged"
    assert same_on_all_ranks(free), f"{name}: ranks disagree on greedy ids"
    # chained decode ends where the host loop ends
    m3 = load()
    for i, t in enumerate(prompt):
        m3.forward(int(t), i, i == P - 1, False)
    first_id = m3.argmax()
    assert first_id == free[0]
    assert m3.decode_chained(first_id, P, G - 1) == free[G - 1]
    # sampled: every id equals the oracle's unless the flip rule explains it
    kw = dict(top_k=20, temp=0.7, top_p=0.9, seed=42)
    s_ref, cands = oracle_sampled(path, prompt, G, kw)
    ms = load(**kw)
    s_ids, _, _, s_lg = ms.generate(prompt, G, forced=s_ref, logits_at=list(range(G)))
    assert same_on_all_ranks(s_ids), f"{name}: ranks disagree on sampled ids"
    flips = check_sampled(s_ids, s_ref, cands, s_lg, 20, 0.7, 0.9, 0.0, uniform_draws(42, G), name)
    assert len(flips) <= 1, f"{name}: sampled flips {flips}"
    # a single-GPU model on rank 0's device runs frames the other ranks never
    # see; the sharded model's exchanges still line up (frame numbers are kept
    # per model, not per device)
    if rank == 0:
        solo = mm.Qwen3Model(path, mm.RunParams(num_iters=4, max_seq_len=P + 5)).set_device("cuda")
        solo.generate(prompt, 4)
        solo.close()
    dist.barrier()
    again, _, _ = m.generate(prompt, G, forced=ref_ids)
    assert list(again) == list(ids), f"{name}: decode after another model's frames differs"
    assert same_on_all_ranks(again)
    for mod in (m, m2, m3, ms):
        assert mod.comm_status() == 0, f"{name}: an exchange wait gave up"
        mod.close()
    dist.barrier()
    return len(events)


def main():
    rank, world, local = env_ranks()
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.cuda.set_device(local)
    mm.init(1, [local])
    device = torch.device("cuda", local)
    # dense models split attention and FFN (tensor parallelism); MoE models split their experts
    names = [n for n in TINY if (TINY[n].n_experts == 0 and TINY[n].n_kv_heads % world == 0
                                 and TINY[n].d_ff % world == 0) or
             (TINY[n].n_experts > 0 and TINY[n].n_experts % world == 0)]
    if rank == 0:
        for n in names:
            tiny_model(n)  # create the files once
    dist.barrier()
    check_allreduce(rank, world, device)
    for n in names:
        ev = check_model(n, rank, world)
        if rank == 0:
            print(f"tp{world} {n}: ok ({ev} tolerance events)", flush=True)
        if TINY[n].n_experts > 0 and TINY[n].n_kv_heads % world == 0:
            # the same MoE model split by experts instead of by rows
            os.environ["MF_MOE_EP"] = "1"
            ev = check_model(n, rank, world)
            os.environ.pop("MF_MOE_EP", None)
            if rank == 0:
                print(f"ep{world} {n}: ok ({ev} tolerance events)", flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
