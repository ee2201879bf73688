"""Source guards (CPU): no source file uses a TMA or bulk load with cluster
multicast (every TMA copy here moves this GPU's own memory, and the
multi-GPU paths must never issue a multicast load from a peer's memory).
The pattern is assembled from pieces so that this file does not contain it."""
import os

from conftest import REPO

MULTICAST_LOAD = ".multi" + "cast::" + "cluster"
EXTS = (".cu", ".cuh", ".cc", ".h", ".py", ".sh", ".tla", ".cfg")
SKIP_DIRS = {".git", "_build", "gpurun_out", "_work", "__pycache__", ".pytest_cache", "baseline"}


def sources():
    for root, dirs, files in os.walk(REPO):
        dirs[:] = [d for d in dirs if d not in SKIP_DIRS]
        for f in files:
            if f.endswith(EXTS) or f == "Makefile":
                yield os.path.join(root, f)


def test_no_cluster_multicast_loads():
    hits = []
    for path in sources():
        text = open(path, encoding="utf-8", errors="replace").read()
        if MULTICAST_LOAD in text:
            hits.append(os.path.relpath(path, REPO))
    assert not hits, hits


def test_tma_copies_exist_and_are_plain_bulk_copies():
    # The TMA paths (NVLS copier warp, local bulk copy) use cp.async.bulk
    # between global and shared memory without a multicast qualifier.
    found = 0
    for path in sources():
        if not path.endswith((".cu", ".cuh")):
            continue
        for line in open(path, encoding="utf-8").read().splitlines():
            if "cp.async.bulk." in line and "wait_group" not in line and "commit_group" not in line:
                found += 1
                assert "multi" + "cast" not in line, line
    assert found >= 4
