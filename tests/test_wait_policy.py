"""CPU: the host wait for a step that ran NCCL kernels (moe_wait.h, used by
moe_api.cu's stream_wait).  NCCL's kernels have no bounded wait of their own,
so the library polls the stream and the communicator, and aborts the
communicator on an asynchronous error or after the time limit.  The policy is
compiled here against fakes of those three calls: no GPU, no NCCL, no peer
that really stops (a GPU test that left an NCCL kernel waiting would be
unbounded)."""
import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_wait_policy_outcomes(tmp_path):
    exe = str(tmp_path / "wait_policy")
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Werror", os.path.join(ROOT, "tests", "wait_policy.cc"),
                    "-o", exe, "-lpthread"], check=True)
    out = subprocess.run([exe], capture_output=True, text=True, timeout=60, check=True).stdout
    got = {}
    for line in out.splitlines():
        name, *kv = line.split()
        got[name] = {k: int(v) for k, v in (x.split("=") for x in kv)}
    # MOE_WAIT_DONE 0, STREAM_ERROR 1, NCCL_ERROR 2, TIMEOUT 3
    assert got["finishes"] == {"outcome": 0, "queries": 5, "aborts": 0}
    assert got["stream_error"] == {"outcome": 1, "queries": 3, "aborts": 0}
    assert got["nccl_error"] == {"outcome": 2, "queries": 4, "aborts": 1}
    assert got["timeout"]["outcome"] == 3 and got["timeout"]["aborts"] == 1
    assert got["timeout"]["queries"] > 10  # it kept polling until the limit
