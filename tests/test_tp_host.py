"""Host side of tensor parallelism on the CPU: the handle exchange over a
world-size-2 gloo group (ordering, validation) and the shard arithmetic
(vocabulary split, head/FFN divisibility) of the host runtime, without a GPU."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from minfer_b200 import tp
from minfer_b200._lib import MF_COMM_HANDLE_BYTES


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class FakeInfo:
    def __init__(self, rank, size):
        self.tp_rank, self.tp_size = rank, size


class FakeModel:
    """Stands in for minfer_b200.model.Qwen3Model: records what connect() passes."""

    def __init__(self, rank, size):
        self.info = FakeInfo(rank, size)
        self.connected = None

    def comm_handle(self):
        return bytes([self.info.tp_rank + 1]) * MF_COMM_HANDLE_BYTES

    def comm_connect(self, handles):
        self.connected = handles


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m = FakeModel(rank, world)
        tp.connect(m)
        ok_order = m.connected == [bytes([r + 1]) * MF_COMM_HANDLE_BYTES for r in range(world)]
        bad = FakeModel((rank + 1) % world, world)  # tp_rank does not match the group rank
        try:
            tp.connect(bad)
            rejected = False
        except ValueError:
            rejected = True
        q.put((rank, ok_order, rejected))
    finally:
        dist.destroy_process_group()


def test_handle_exchange_gloo_world2():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=5) for _ in range(world))
    assert res == [(0, True, True), (1, True, True)]


def test_env_ranks_default(monkeypatch):
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        monkeypatch.delenv(k, raising=False)
    assert tp.env_ranks() == (0, 1, 0)
    monkeypatch.setenv("RANK", "3")
    monkeypatch.setenv("WORLD_SIZE", "8")
    monkeypatch.setenv("LOCAL_RANK", "3")
    assert tp.env_ranks() == (3, 8, 3)


@pytest.mark.parametrize("size", [1, 2, 4, 8])
def test_shard_load_splits(size):
    """Every rank of a tp_size split loads (CPU side only) and reports its
    position; KV heads that do not divide are refused with a message."""
    import ctypes as C

    from conftest import tiny_model
    from minfer_b200._lib import MF_OK, host_lib, last_error, mf_model_info, mf_run_params

    rp = mf_run_params(8, 64, 1, 0.0, 1.0, 0.0, 0.0, 0)
    for rank in range(size):
        m = C.c_void_p()
        rc = host_lib().mf_model_load_tp(tiny_model("tiny-tp8").encode(), C.byref(rp), 0, rank, size, C.byref(m))
        assert rc == MF_OK, last_error()
        info = mf_model_info()
        assert host_lib().mf_model_info_get(m, C.byref(info)) == MF_OK
        assert (info.tp_rank, info.tp_size) == (rank, size)
        host_lib().mf_model_free(m)
    m = C.c_void_p()
    rc = host_lib().mf_model_load_tp(tiny_model("tiny-bf16").encode(), C.byref(rp), 0, 0, 4, C.byref(m))
    assert rc != MF_OK and "n_kv_heads" in last_error()
    # the MoE model (2 KV heads, 16 experts): rows split at 2 ranks, experts at 4, 3 divides neither
    rc = host_lib().mf_model_load_tp(tiny_model("tiny-moe").encode(), C.byref(rp), 0, 1, 2, C.byref(m))
    assert rc == MF_OK, last_error()
    info = mf_model_info()
    assert host_lib().mf_model_info_get(m, C.byref(info)) == MF_OK and (info.tp_rank, info.tp_size) == (1, 2)
    host_lib().mf_model_free(m)
    rc = host_lib().mf_model_load_tp(tiny_model("tiny-moe").encode(), C.byref(rp), 0, 0, 3, C.byref(m))
    assert rc != MF_OK and "expert_count" in last_error()
    rc = host_lib().mf_model_load_tp(tiny_model("tiny-bf16").encode(), C.byref(rp), 0, 2, 2, C.byref(m))
    assert rc != MF_OK


def _expert_parallel(path, rank, size):
    import ctypes as C

    from minfer_b200._lib import MF_OK, host_lib, last_error, mf_model_info, mf_run_params

    rp = mf_run_params(8, 64, 1, 0.0, 1.0, 0.0, 0.0, 0)
    m = C.c_void_p()
    rc = host_lib().mf_model_load_tp(path.encode(), C.byref(rp), 0, rank, size, C.byref(m))
    assert rc == MF_OK, last_error()
    info = mf_model_info()
    assert host_lib().mf_model_info_get(m, C.byref(info)) == MF_OK
    host_lib().mf_model_free(m)
    return info.expert_parallel


def test_moe_split_choice(monkeypatch):
    """How a MoE model splits over the ranks (CPU side, at load): by FFN rows
    inside every expert (attention by KV-head group) when the KV heads divide
    over the ranks, else by experts; MF_MOE_EP=1 forces experts. The 4-KV-head
    shape is 30B-A3B's head layout: rows at 2 and 4 ranks, experts at 8."""
    from conftest import model_dir, tiny_model
    from minfer_b200.gguf_synth import Qwen3Shape, ensure_gguf

    kv2 = tiny_model("tiny-moe")
    kv4 = ensure_gguf(model_dir() / "tiny-moe-kv4.gguf",
                      Qwen3Shape(2, 256, 8, 4, 128, 128, 1024, "bf16", False, 16, 4, seed=108))
    for path, size, want in [(kv2, 2, 0), (kv2, 4, 1), (kv2, 8, 1), (kv4, 2, 0), (kv4, 4, 0), (kv4, 8, 1)]:
        for rank in range(size):
            assert _expert_parallel(path, rank, size) == want, (path, size, rank)
    monkeypatch.setenv("MF_MOE_EP", "1")
    assert _expert_parallel(kv4, 0, 4) == 1
