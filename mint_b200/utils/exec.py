"""Run untrusted snippets with captured stdout/stderr and a SIGALRM time limit (mint/utils/exec.py:9-67)."""

from __future__ import annotations

import io
import signal
import sys
from collections.abc import Iterator
from contextlib import contextmanager
from typing import NamedTuple, Never


class ExecutionResult(NamedTuple):
    success: bool
    output: str = ""
    error: str = ""


class TimeoutHandlerError(Exception):
    pass


def timeout_handler(signum, frame) -> Never:  # noqa: ANN001, ARG001
    raise TimeoutHandlerError("Code execution timed out")


@contextmanager
def time_limit(seconds: int) -> Iterator[None]:
    previous = signal.signal(signal.SIGALRM, timeout_handler)
    signal.alarm(seconds)
    try:
        yield
    finally:
        signal.alarm(0)
        signal.signal(signal.SIGALRM, previous)


def execute_code(code: str, timeout: int = 5) -> ExecutionResult:
    out, err = io.StringIO(), io.StringIO()
    saved = sys.stdout, sys.stderr
    try:
        sys.stdout, sys.stderr = out, err
        with time_limit(timeout):
            exec(code, {"__builtins__": __builtins__})  # noqa: S102
        error = err.getvalue()
        return ExecutionResult(success=not error, output=out.getvalue(), error=error)
    except TimeoutHandlerError as exc:
        return ExecutionResult(success=False, output=out.getvalue(), error=f"Timeout: {exc!s}")
    except Exception as exc:  # noqa: BLE001
        return ExecutionResult(success=False, output=out.getvalue(), error=f"{type(exc).__name__}: {exc!s}")
    finally:
        sys.stdout, sys.stderr = saved
