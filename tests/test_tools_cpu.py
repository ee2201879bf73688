"""CPU checks of the measurement and stress tools' pure parts: nccl-tests
bus-bandwidth factors, size parsing, the size ladder, and the stress
harness's case generators (thresholds read through the library's policy
parser, boundary cases at -1/0/+1 element, odd tails that fill no vector)."""
import pytest

from scc26_nccl_shim_b200.parallel import stress, sweep


def test_busbw_factors():
    s = 1.0
    assert sweep.busbw("allreduce", 10**9, s, 8) == pytest.approx(2 * 7 / 8)
    assert sweep.busbw("allgather", 10**9, s, 8) == pytest.approx(7 / 8)
    assert sweep.busbw("reducescatter", 10**9, s, 4) == pytest.approx(3 / 4)
    assert sweep.busbw("broadcast", 10**9, s, 8) == pytest.approx(1.0)
    assert sweep.busbw("allreduce", 10**9, s, 1) == pytest.approx(1.0)  # one GPU: algbw


def test_size_parsing_and_ladder():
    assert sweep.parse_size("8") == 8
    assert sweep.parse_size("64K") == 64 << 10
    assert sweep.parse_size("8G") == 8 << 30
    assert sweep.parse_size("512MiB") == 512 << 20
    assert list(sweep.sizes(8, 512, 4)) == [8, 32, 128, 512]


def test_stress_cases(monkeypatch):
    monkeypatch.setenv("NCCL_B200_AR_MIN", "4M")
    thr = stress.thresholds()
    assert thr["allreduce"] == 4 << 20 and thr["allgather"] == 32 << 20
    b = stress.boundary_cases(4, thr)
    counts = {c.name: c.count for c in b}
    assert counts["bnd_allreduce_+0"] == (4 << 20) // 4
    assert counts["bnd_allreduce_-1"] == (4 << 20) // 4 - 1
    assert counts["bnd_allgather_+1"] == (32 << 20) // 4 // 4 + 1
    cases = stress.standard_cases(4, scale=4)
    names = {c.name for c in cases}
    for kind in ("allreduce", "allgather", "reducescatter", "broadcast"):
        assert f"{kind}_float32_oop" in names and f"{kind}_bfloat16_ip" in names
        assert f"{kind}_float32_odd" in names
    rs = [c for c in cases if c.kind == "reducescatter"]
    assert all(c.count % 8 == 0 for c in rs)  # 16-byte slots for every dtype used
    assert any(c.op == "max" for c in cases)
