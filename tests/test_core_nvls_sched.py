"""The NVLS AllReduce round schedule (src/core/nvls_sched.h), shared by the
kernel and the host's progress-step count: the rounds partition the message
in order, none exceeds the scratch round, and the ramped schedule starts and
ends with short rounds."""
import pytest

from scc26_nccl_shim_b200 import _core as c

MiB = 1 << 20


@pytest.mark.parametrize("ramp", [False, True])
@pytest.mark.parametrize("R", [4 * MiB, 64 * MiB, 256 * MiB, 9472 * 4])
def test_rounds_partition_the_message(R, ramp):
    for nbytes in (16, 32, R - 16, R, R + 16, 4 * R - 32, 4 * R, 4 * R + 32, 5 * R + R // 16,
                   7 * R + 48, 32 * R, 33 * R - 16):
        rounds = c.nvls_ar_rounds(nbytes, R, ramp)
        at = 0
        for base, ln in rounds:
            assert base == at and 0 < ln <= R, (nbytes, R, rounds)
            at += ln
        assert at == nbytes


def test_ramp_shape():
    R = 256 * MiB
    q = R // 8
    rounds = c.nvls_ar_rounds(32 * R, R, True)
    lens = [ln for _, ln in rounds]
    assert lens[:4] == [q, q, 2 * q, 4 * q] and lens[-4:] == [4 * q, 2 * q, q, q]
    assert all(ln == R for ln in lens[4:-4]) and len(lens) == 8 + 30
    # Below 4R the schedule is uniform.
    assert [ln for _, ln in c.nvls_ar_rounds(4 * R - 32, R, True)] == [R, R, R, R - 32]
    assert c.nvls_ar_rounds(8 * R, R, False) == [(i * R, R) for i in range(8)]


def test_nvls_shape_packs_and_unpacks():
    """A tuned NVLS kernel shape travels as one int (calibration cache):
    every field reads back, and the largest shape stays below INT_MAX."""
    import ctypes as C
    L = c.lib()
    out = (C.c_int * 5)()
    for shape in [(0, 0, 0, 0, 0), (608, 4, 0, 0, 0), (608, 8, 0, 0, 2), (512, 8, 128, 2, 2), (1999, 9, 9999, 2, 2)]:
        v = L.nb_nvls_shape(*shape, out)
        assert 0 <= v < 2 ** 31 - 1 and tuple(out) == shape, (shape, v, tuple(out))
