"""Run a code snippet in a separate Python process with captured output and a wall-clock limit.

Used to grade generated programs (HumanEval). The reference runs the snippet with ``exec`` inside
the trainer process under a SIGALRM alarm (mint/utils/exec.py:9-67), which only works on the main
thread and lets the snippet touch the trainer's state. Here every snippet runs in its own
interpreter (``python -I -c``: isolated mode, no user site, no environment-driven imports) in a
new session, with stdin closed; on timeout the whole process group is killed, so a snippet that
forks or loops forever cannot outlive its limit. The result type is the reference's.
"""

from __future__ import annotations

import os
import signal
import subprocess
import sys
from typing import NamedTuple


class ExecutionResult(NamedTuple):
    success: bool
    output: str = ""
    error: str = ""


def execute_code(code: str, timeout: int | float = 5) -> ExecutionResult:
    """Run ``code`` and report ``success`` when it exits 0 and wrote nothing to stderr."""
    try:
        proc = subprocess.Popen([sys.executable, "-I", "-c", code], stdin=subprocess.DEVNULL,
                                stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True, start_new_session=True)
    except OSError as exc:
        return ExecutionResult(success=False, error=f"{type(exc).__name__}: {exc}")
    try:
        out, err = proc.communicate(timeout=timeout)
    except subprocess.TimeoutExpired:
        _kill_group(proc)
        out, err = proc.communicate()
        return ExecutionResult(success=False, output=out or "", error=f"Timeout: code execution exceeded {timeout} s")
    if proc.returncode != 0:
        tail = err.strip().splitlines()[-1] if err.strip() else f"exit code {proc.returncode}"
        return ExecutionResult(success=False, output=out, error=tail)
    return ExecutionResult(success=not err, output=out, error=err)


def _kill_group(proc: subprocess.Popen) -> None:
    try:
        os.killpg(proc.pid, signal.SIGKILL)  # the snippet's own process group only (new session)
    except (ProcessLookupError, PermissionError):
        proc.kill()
