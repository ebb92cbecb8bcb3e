"""Failure handling on CPU gloo ranks (no GPU is involved, so nothing here can fault a GPU).

* SIGINT on one rank: the interrupt flag is MAX-reduced at the next step boundary, every rank stops
  there and takes part in the collective forced checkpoint; resuming from it reproduces the
  parameters of an uninterrupted run.
* A rank that dies between steps: the survivor's next collective fails within the process-group
  timeout and the process exits with an error instead of hanging.
"""

import socket
import subprocess
import sys
import time
from pathlib import Path

import torch

WORKER = Path(__file__).with_name("fault_worker.py")


def _port() -> str:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return str(s.getsockname()[1])


def _run(mode: str, work: Path, timeout: float = 180.0) -> list[subprocess.CompletedProcess]:
    port = _port()
    procs = [subprocess.Popen([sys.executable, str(WORKER), mode, str(r), "2", port, str(work)],
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True) for r in range(2)]
    out = []
    deadline = time.monotonic() + timeout
    for p in procs:
        try:
            text, _ = p.communicate(timeout=max(1.0, deadline - time.monotonic()))
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise AssertionError(f"{mode}: a rank did not exit within {timeout} s") from None
        out.append(subprocess.CompletedProcess(p.args, p.returncode, text, ""))
    return out


def test_sigint_checkpoint_and_resume(tmp_path):
    full = _run("full", tmp_path / "a")
    assert all(r.returncode == 0 for r in full), full[0].stdout[-3000:] + full[1].stdout[-3000:]
    work = tmp_path / "b"
    stop = _run("sigint", work)
    assert all(r.returncode == 0 for r in stop), stop[0].stdout[-3000:] + stop[1].stdout[-3000:]
    ckpt = torch.load(work / "ckpt" / "checkpoint_latest.pt", map_location="cpu", weights_only=False)
    assert ckpt["step"] == 3  # the step boundary after the signal, on both ranks
    assert set(ckpt["dataloader_state"]["per_rank"]) == {0, 1}
    res = _run("resume", work)
    assert all(r.returncode == 0 for r in res), res[0].stdout[-3000:] + res[1].stdout[-3000:]
    assert "resumed at step 3" in res[0].stdout
    a = torch.load(tmp_path / "a" / "final_full.pt")
    b = torch.load(work / "final_resume.pt")
    for k in a:
        assert torch.allclose(a[k], b[k], rtol=1e-5, atol=1e-7), k


def test_dead_rank_fails_survivor_collective(tmp_path):
    t0 = time.monotonic()
    res = _run("die", tmp_path, timeout=120.0)
    assert res[1].returncode == 0  # the rank that left
    assert res[0].returncode != 0, res[0].stdout[-3000:]
    assert "die done" not in res[0].stdout
    assert time.monotonic() - t0 < 120.0
