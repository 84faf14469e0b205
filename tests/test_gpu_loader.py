"""The GGUF -> device loader path: uploads through the pinned staging ring
(32 MiB buffers filled by host threads) land byte for byte, for sizes below,
at and across the ring's buffer size and at unaligned offsets; the strided
upload that lays weight rows out (gate/up interleaving, tensor-parallel
column shards) places every run and touches nothing else. (That whole models
load exactly is shown by the parity tests, whose logits need every weight.)"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

STAGE = 32 << 20


@pytest.fixture(scope="module")
def lib(gpu):
    from minfer_b200._lib import cuda_lib

    return cuda_lib()


def _buf(lib, nbytes):
    from minfer_b200._lib import check

    b = C.c_void_p()
    check(lib.mf_alloc(nbytes, 0, C.byref(b)))
    return b


@pytest.mark.parametrize("nbytes", [1, 4095, STAGE - 16, STAGE, STAGE + 1, 3 * STAGE + 12345])
def test_upload_and_read_round_trip(lib, nbytes):
    from minfer_b200._lib import check

    rng = np.random.default_rng(nbytes % 1000)
    src = rng.integers(0, 256, nbytes, dtype=np.uint8)
    b = C.c_void_p()
    check(lib.mf_upload(src.ctypes.data, nbytes, 0, C.byref(b)))
    back = np.zeros(nbytes, np.uint8)
    check(lib.mf_read(b, 0, back.ctypes.data, nbytes))
    assert np.array_equal(src, back)
    # a write at an odd offset replaces exactly its range
    if nbytes > 1000:
        patch = rng.integers(0, 256, nbytes // 3, dtype=np.uint8)
        off = 777
        check(lib.mf_write(b, off, patch.ctypes.data, patch.size))
        check(lib.mf_read(b, 0, back.ctypes.data, nbytes))
        want = src.copy()
        want[off:off + patch.size] = patch
        assert np.array_equal(want, back)
    lib.mf_release(b)


@pytest.mark.parametrize("rows,width,src_pitch,dst_pitch", [(7, 48, 64, 96), (3000, 4096, 8192, 4096 * 2),
                                                            (20000, 2048, 2048, 4096)])
def test_strided_upload_places_every_run(lib, rows, width, src_pitch, dst_pitch):
    from minfer_b200._lib import check

    rng = np.random.default_rng(rows)
    host = rng.integers(0, 256, rows * src_pitch, dtype=np.uint8)
    total = 64 + rows * dst_pitch
    b = _buf(lib, total)
    check(lib.mf_write_2d(b, 64, dst_pitch, host.ctypes.data, src_pitch, width, rows))
    back = np.zeros(total, np.uint8)
    check(lib.mf_read(b, 0, back.ctypes.data, total))
    runs = back[64:].reshape(rows, dst_pitch)
    assert np.array_equal(runs[:, :width], host.reshape(rows, src_pitch)[:, :width])
    assert not runs[:, width:].any() and not back[:64].any()  # nothing outside the runs (zero-filled alloc)
    lib.mf_release(b)

