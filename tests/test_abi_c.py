"""A C program written against the reference's runtime and device-owner
interfaces (tests/abi_c/owner_abi.c), compiled and linked against
libchelis_cuda alone: the reference-named symbols resolve, the metadata-plan
and host-tensor stand-ins do the runtime's arithmetic, misuse fails the way
the runtime fails, and (on a GPU) the owner round trip and the host-array
matmul entry give the right results."""
import os
import shutil
import subprocess

import pytest

from chelis_b200 import lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "abi_c", "owner_abi.c")


@pytest.fixture(scope="module")
def owner_abi(tmp_path_factory):
    cc = shutil.which("gcc") or shutil.which("cc")
    if not cc:
        pytest.skip("no C compiler")
    L.load()  # the library must exist (built in-tree)
    exe = str(tmp_path_factory.mktemp("abi_c") / "owner_abi")
    libdir = os.path.dirname(L.LIB_PATH)
    subprocess.run([cc, "-std=c99", "-Wall", "-Werror", "-O1", "-I", os.path.join(ROOT, "include"),
                    SRC, "-o", exe, "-L", libdir, "-l:libchelis_cuda.so",
                    f"-Wl,-rpath,{libdir}", "-lm"], check=True)
    return exe


def run(exe, mode):
    return subprocess.run([exe, mode], capture_output=True, text=True, timeout=120)


def test_plan_and_host_tensor_arithmetic(owner_abi):
    r = run(owner_abi, "plan")
    assert r.returncode == 0, r.stderr
    assert "plan ok" in r.stdout


def test_status_forms_report_codes(owner_abi):
    r = run(owner_abi, "status")
    assert r.returncode == 0, r.stderr


@pytest.mark.parametrize("mode", ["trap-rank", "trap-view"])
def test_metadata_errors_trap_like_the_runtime(owner_abi, mode):
    # chelis_runtime.h:127-130: the trap line on stderr, then exit(1)
    r = run(owner_abi, mode)
    assert r.returncode == 1
    assert "numeric trap: domain in metadata_plan at i64" in r.stderr


@pytest.mark.gpu
def test_owner_round_trip_and_host_array_matmul(owner_abi):
    r = run(owner_abi, "gpu")
    assert r.returncode == 0, r.stdout + r.stderr
    assert "gpu ok" in r.stdout
