"""The tensor-parallel watchdog on the host (no GPU): the bounded wait of
vox_watchdog.h compiled with g++ against fakes of the CUDA stream query, the
NCCL asynchronous-error poll and the communicator abort.  A stopped rank
(a stream that never goes idle) ends in an abort after the timeout; an
asynchronous error aborts at once; an idle stream returns without one."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_watchdog_scenarios(tmp_path):
    exe = str(tmp_path / "watchdog_check")
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "voxtral-rust_b200", "csrc"),
                    os.path.join(ROOT, "tests", "watchdog_check.cpp"), "-o", exe], check=True)
    out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout.split("\n")
    res = {ln.split()[0]: (int(ln.split()[1]), int(ln.split()[2]), float(ln.split()[3])) for ln in out if ln}
    # kWatchdogIdle 0, kWatchdogAsyncError 1, kWatchdogTimeout 2, kWatchdogStreamError 3
    assert res["idle_at_once"][:2] == (0, 0)
    assert res["idle_after_polls"][:2] == (0, 0)
    assert res["async_error"][:2] == (1, 1)
    r, aborts, ms = res["rank_stopped_timeout"]
    assert (r, aborts) == (2, 1) and 300 <= ms < 5000
    assert res["stream_error"][:2] == (3, 0)
