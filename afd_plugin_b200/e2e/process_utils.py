"""Launching and tearing down server process groups for end-to-end runs.

Every server is started as the leader of a new session, so it and everything
it spawns (``torch.distributed.run`` and its ranks) share one process group
that belongs to this runner alone.  Teardown signals that group: SIGTERM
first, SIGKILL for whatever is still there after a grace period -- the
escalation of the reference's ``tests/e2e/process_utils.py:35-160``, which
uses pidfds for the same purpose.
"""

from __future__ import annotations

import os
import signal
import subprocess
import time
from dataclasses import dataclass, field

import requests


@dataclass
class ServerProcess:
    cmd: list[str]
    proc: subprocess.Popen
    log_path: str | None = None
    started: float = field(default_factory=time.monotonic)

    @property
    def pgid(self) -> int:
        return self.proc.pid  # session leader: its pid is the group id

    def log_tail(self, n: int = 40) -> str:
        if not self.log_path or not os.path.exists(self.log_path):
            return ""
        with open(self.log_path, errors="replace") as fh:
            return "".join(fh.readlines()[-n:])


def start_server(cmd: list[str], *, env: dict[str, str] | None = None, log_path: str | None = None,
                 cwd: str | None = None) -> ServerProcess:
    out = open(log_path, "w") if log_path else subprocess.DEVNULL  # noqa: SIM115 - owned by the child
    try:
        proc = subprocess.Popen(cmd, env=env, cwd=cwd, stdout=out, stderr=subprocess.STDOUT,
                                stdin=subprocess.DEVNULL, start_new_session=True)
    finally:
        if log_path:
            out.close()
    return ServerProcess(cmd, proc, log_path)


def group_alive(pgid: int) -> bool:
    try:
        os.killpg(pgid, 0)
    except ProcessLookupError:
        return False
    except PermissionError:
        return True
    return True


def stop_server(server: ServerProcess, *, term_timeout_s: float = 20.0, kill_timeout_s: float = 10.0) -> str:
    """End the server's whole process group; returns "exited", "terminated" or "killed"."""
    pgid = server.pgid
    if server.proc.poll() is not None and not group_alive(pgid):
        return "exited"
    how = "terminated"
    try:
        os.killpg(pgid, signal.SIGTERM)
    except ProcessLookupError:
        pass
    deadline = time.monotonic() + term_timeout_s
    while time.monotonic() < deadline and (server.proc.poll() is None or group_alive(pgid)):
        time.sleep(0.05)
    if server.proc.poll() is None or group_alive(pgid):
        how = "killed"
        try:
            os.killpg(pgid, signal.SIGKILL)
        except ProcessLookupError:
            pass
        try:
            server.proc.wait(kill_timeout_s)
        except subprocess.TimeoutExpired:
            pass
        deadline = time.monotonic() + kill_timeout_s
        while time.monotonic() < deadline and group_alive(pgid):
            time.sleep(0.05)
    return how


def wait_for_health(server: ServerProcess, url: str, *, timeout_s: float = 600.0, interval_s: float = 0.5) -> float:
    """Poll ``url`` + ``/health`` until it answers 200; returns the seconds waited.

    Raises as soon as the server's process exits (with the tail of its log)
    or when ``timeout_s`` passes.
    """
    t0 = time.monotonic()
    while True:
        code = server.proc.poll()
        if code is not None:
            raise RuntimeError(f"server exited with code {code} before it was healthy:\n{server.log_tail()}")
        try:
            if requests.get(url.rstrip("/") + "/health", timeout=5).status_code == 200:
                return time.monotonic() - t0
        except requests.RequestException:
            pass
        if time.monotonic() - t0 > timeout_s:
            raise TimeoutError(f"server at {url} not healthy after {timeout_s:.0f} s:\n{server.log_tail()}")
        time.sleep(interval_s)


__all__ = ["ServerProcess", "group_alive", "start_server", "stop_server", "wait_for_health"]
