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
