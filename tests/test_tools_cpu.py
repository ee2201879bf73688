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


def test_pipeline_and_big_cases():
    env = {"NCCL_B200_NVLS_ROUND": "4M", "NCCL_B200_RING_CHUNK": "32K", "NCCL_B200_HOST_PIECE": "256K"}
    cases = stress.pipeline_cases(4, env, 148)
    names = {c.name for c in cases}
    for edge in ("nvls_round_ar", "nvls_part_rs", "ring_step_bc", "push_round_rs", "host_piece_ar"):
        assert {f"edge_{edge}_-8", f"edge_{edge}_+0", f"edge_{edge}_+8"} <= names, edge
    by = {c.name: c for c in cases}
    assert by["edge_nvls_round_ar_+0"].count * 4 == 4 << 20
    assert by["edge_ring_step_bc_+8"].count * 4 == 32 * 1024 * 148 + 32
    assert all(c.count % 4 == 0 for c in cases if c.kind == "reducescatter")
    big = {c.name: c for c in stress.big_cases(8)}
    assert big["cap_allreduce_at"].count * 4 == 8 << 30
    assert big["cap_allreduce_above"].count * 4 == (8 << 30) + 4
    assert big["big_2g_allreduce_-1"].count == (2 << 30) // 4 - 1


def test_fold_reference_matches_ops():
    import torch
    x = [torch.tensor([1.0, -2.0, 3.0]), torch.tensor([4.0, 5.0, -6.0]), torch.tensor([2.0, 2.0, 2.0])]
    assert stress.fold_ref(x, "sum", torch.float32, 3, 0.5).tolist() == [7.0, 5.0, -1.0]
    assert stress.fold_ref(x, "prod", torch.float32, 3, 0.5).tolist() == [8.0, -20.0, -36.0]
    assert stress.fold_ref(x, "min", torch.float32, 3, 0.5).tolist() == [1.0, -2.0, -6.0]
    assert stress.fold_ref(x, "premulsum", torch.float32, 3, 0.5).tolist() == [3.5, 2.5, -0.5]
    assert stress.fold_ref(x, "avg", torch.float32, 3, 0.5).tolist() == pytest.approx([7 / 3, 5 / 3, -1 / 3])
    xi = [torch.tensor([7, -7], dtype=torch.int32), torch.tensor([0, 0], dtype=torch.int32)]
    assert stress.fold_ref(xi, "avg", torch.int32, 2, 1.0).tolist() == [3, -3]  # truncation toward zero


def test_mixed_workload_draws():
    import random
    from scc26_nccl_shim_b200.parallel import mixed
    calls = mixed.draw_calls(random.Random(0), 64, 8, 4096, 1 << 30, unsupported=True)
    assert len(calls) == 64 and any(k == "send_recv" for k, *_ in calls)
    assert {k for k, *_ in calls} >= {"allreduce", "allgather", "reducescatter", "broadcast"}
    for kind, dtype, op, count in calls:
        assert count >= 8 and count % 8 == 0
        assert op == "sum" or kind in ("allreduce", "reducescatter")
    eligible = mixed.draw_calls(random.Random(1), 64, 8, 64 << 20, 1 << 30, unsupported=False)
    assert not any(k == "send_recv" for k, *_ in eligible)
