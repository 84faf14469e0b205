"""Tensor parallelism on the GPU.

* test_tp_parity: tests/tp_worker.py under torch.distributed.run, one process
  per GPU (2 by default, MF_TP_TEST_RANKS up to 8); skipped with one GPU.
* test_exchange_wait_times_out: one GPU, a rank "connected" to a peer that
  never sends (its own handle in the peer's place): the wait gives up after
  MF_COMM_TIMEOUT_MS, sets the status bit, and the stream stays usable.
"""
import ctypes as C
import os
import socket
import subprocess
import sys
import time
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_tp_parity(gpu):
    n = torch.cuda.device_count()
    want = int(os.environ.get("MF_TP_TEST_RANKS", "2"))
    if n < 2:
        pytest.skip("tensor parallelism needs at least 2 GPUs")
    ranks = max(2, min(want, n))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "900", sys.executable, "-m", "torch.distributed.run", "--nnodes", "1",
           "--nproc-per-node", str(ranks), "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           str(ROOT / "tests" / "tp_worker.py")]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    print(r.stdout[-4000:])
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-6000:]
    assert f"tp{ranks} tiny-tp8: ok" in r.stdout


def test_exchange_wait_times_out(gpu, monkeypatch):
    from minfer_b200 import ops
    from minfer_b200._lib import MF_COMM_HANDLE_BYTES, MF_OK, check, cuda_lib

    monkeypatch.setenv("MF_COMM_TIMEOUT_MS", "200")
    lib = cuda_lib()
    comm = C.c_void_p()
    n = 256
    check(lib.mf_comm_create(0, 0, 2, n, 0, C.byref(comm)))
    try:
        h = (C.c_char * MF_COMM_HANDLE_BYTES)()
        check(lib.mf_comm_handle(comm, h, MF_COMM_HANDLE_BYTES))
        blob = bytes(h) * 2  # rank 1 = this rank's own region: it never sends
        check(lib.mf_comm_connect(comm, C.create_string_buffer(blob, len(blob)), len(blob)))
        x = torch.ones(n, device=gpu)
        out = torch.zeros(n, device=gpu)
        st = torch.tensor([0, 0, 0, 0, 1, 0, 0, 0], dtype=torch.int32, device=gpu)
        t0 = time.time()
        check(lib.mf_allreduce(C.c_void_p(out.data_ptr()), C.c_void_p(x.data_ptr()), C.c_void_p(x.data_ptr()), n,
                               comm, 0, C.c_void_p(st.data_ptr()), C.c_void_p(ops._stream())))
        st = C.c_int()
        assert lib.mf_comm_status(comm, C.byref(st), 1) == MF_OK
        dt = time.time() - t0
        assert st.value & 1, "the wait for the silent peer should have given up"
        assert 0.15 < dt < 10, dt
        # status was cleared, and the device still works
        assert lib.mf_comm_status(comm, C.byref(st), 1) == MF_OK and st.value == 0
        y = (x * 3).sum().item()
        assert y == 3 * n
    finally:
        lib.mf_comm_destroy(comm)


def test_model_timeout_is_an_error(gpu, monkeypatch):
    """A model-level frame whose exchange wait gave up fails with MF_E_TIMEOUT
    (forward, chained decode, generate) instead of returning ids: rank 0 of a
    2-rank model is connected to a peer that never sends (its own handle in
    the peer's place)."""
    from conftest import tiny_model
    from minfer_b200 import model as mm
    from minfer_b200._lib import MF_E_TIMEOUT, MinferError

    monkeypatch.setenv("MF_COMM_TIMEOUT_MS", "50")
    m = mm.Qwen3Model(tiny_model("tiny-tp8"), mm.RunParams(num_iters=4, max_seq_len=16), tp_rank=0,
                      tp_size=2).set_device("cuda")
    h = m.comm_handle()
    m.comm_connect([h, h])
    with pytest.raises(MinferError) as e:
        m.forward(3, 0, True, False)
    assert e.value.code == MF_E_TIMEOUT, e.value
    assert m.comm_status() != 0  # the bits stay readable (and are cleared by reading them)
    with pytest.raises(MinferError) as e:
        m.decode_chained(3, 1, 2)
    assert e.value.code == MF_E_TIMEOUT, e.value
    with pytest.raises(MinferError) as e:
        m.generate(np.array([1, 2, 3], np.uint32), 2, token_prefill=True)
    assert e.value.code == MF_E_TIMEOUT, e.value
    m.close()
    # the device is still usable
    assert (torch.ones(8, device=gpu) * 2).sum().item() == 16
