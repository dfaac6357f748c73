"""Failure detection of the tensor-parallel communicators, on the CPU.

The watchdog logic that mllm_comm_* runs against NCCL (mllm_b200/csrc/comm_watchdog.h) is
compiled here against fake operations -- a clock the test moves, events the test completes, an
asynchronous error the test raises -- and checked for: collectives completing in time, a
collective that never completes (a peer that never joins) aborted at its deadline, an
asynchronous error aborted at once, an abort on request, and a polling thread racing a
tracking thread.  No GPU and no NCCL are involved."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def check_binary(tmp_path_factory):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.fail("g++ is required for the watchdog check")
    out = str(tmp_path_factory.mktemp("wd") / "comm_watchdog_check")
    subprocess.run([gxx, "-std=c++17", "-O1", "-pthread", "-I", os.path.join(ROOT, "mllm_b200", "csrc"),
                    os.path.join(ROOT, "tests", "native", "comm_watchdog_check.cpp"), "-o", out], check=True)
    return out


def test_watchdog_scenarios(check_binary):
    r = subprocess.run([check_binary], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    lines = r.stdout.split()
    for name in ("healthy", "timeout", "per_collective_deadline", "async_error", "abort_on_request", "threads"):
        assert name in lines, r.stdout
