"""Child processes tied to this process (reference: core/proc_tree.py:25-242).

``spawn`` starts a child in its own process group that receives SIGTERM when
the parent dies (PR_SET_PDEATHSIG on Linux), so serving workers never outlive
the server; ``stop`` terminates a child's whole group with a timeout."""

from __future__ import annotations

import ctypes
import os
import signal
import subprocess

_PR_SET_PDEATHSIG = 1


def _child_setup():
    os.setsid()
    try:
        libc = ctypes.CDLL("libc.so.6", use_errno=True)
        libc.prctl(_PR_SET_PDEATHSIG, signal.SIGTERM)
    except OSError:
        pass


def spawn(cmd, env=None, cwd=None, stdout=None, stderr=None) -> subprocess.Popen:
    return subprocess.Popen(cmd, env=env, cwd=cwd, stdout=stdout, stderr=stderr, preexec_fn=_child_setup)


def stop(proc: subprocess.Popen, timeout: float = 10.0) -> int:
    if proc.poll() is not None:
        return proc.returncode
    try:
        os.killpg(proc.pid, signal.SIGTERM)
    except ProcessLookupError:
        return proc.poll()
    try:
        return proc.wait(timeout=timeout)
    except subprocess.TimeoutExpired:
        os.killpg(proc.pid, signal.SIGKILL)
        return proc.wait(timeout=timeout)
