"""The blocking-communicator check of the init interposers, through the
interposer library itself on the CPU (no GPU needed to load it): only
blocking communicators (NCCL_COMM_BLOCKING unset or 1, config blocking 1 or
left undefined) with a well-formed ncclConfig_t (its size covers `blocking`,
magic 0xcafebeef, version in the supported range) may be driven by the
interposer. Counterpart: shim.cu:1461-1470 of the reference, which accepts
versions 2.14-2.28.3 only."""
import ctypes as C
import os
import subprocess
import sys

from conftest import REPO

CHILD = r"""
import ctypes as C, sys
sys.path.insert(0, {repo!r})
from scc26_nccl_shim_b200 import LIB_PATH, real_nccl_path
C.CDLL(real_nccl_path(), mode=C.RTLD_GLOBAL)
L = C.CDLL(LIB_PATH, mode=C.RTLD_GLOBAL)
L.nb_blocking_config.argtypes = [C.c_int, C.c_size_t, C.c_uint, C.c_uint, C.c_int]
UNDEF = -2147483648
V = L.nb_nccl_version() or 22809
cases = [(0, 0, 0, 0, 0), (1, 0, 0xcafebeef, V, 1), (1, 0, 0xcafebeef, V, UNDEF),
         (1, 0, 0xcafebeef, V, 0), (1, 0, 0xdeadbeef, V, 1), (1, 0, 0xcafebeef, 21000, 1),
         (1, 0, 0xcafebeef, 23500, 1), (1, 8, 0xcafebeef, V, 1)]
print(" ".join(str(L.nb_blocking_config(*c)) for c in cases))
"""


def run(env_extra):
    env = dict(os.environ, **env_extra)
    env.pop("LD_PRELOAD", None)
    r = subprocess.run([sys.executable, "-c", CHILD.format(repo=REPO)], env=env, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    return r.stdout.split()[-8:]


def test_blocking_configuration():
    # no config, blocking 1, undefined, non-blocking, bad magic, too old, too new, truncated
    assert run({}) == ["1", "1", "1", "0", "0", "0", "0", "0"]


def test_nonblocking_environment_disables_the_interposer():
    env = {"NCCL_COMM_BLOCKING": "0"}
    assert run(env) == ["0"] * 8
