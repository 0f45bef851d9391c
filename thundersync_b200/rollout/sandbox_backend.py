"""Which container runtime a site's sandboxes run on (C53).

Docker when this user's Docker daemon answers, udocker otherwise. ``auto``
applies that rule; an explicit ``docker`` or ``udocker`` request is honoured
only when that runtime is usable and is refused otherwise — never swapped for
the other. Resolve once per site and hand the result to every process
(reference: src/thundersync/rollout/sandbox_backend.py:1-239; the JSON record
schema name is kept so tooling that reads it still does).

``python -m thundersync_b200.rollout.sandbox_backend --requested auto`` prints
the resolution record.
"""

from __future__ import annotations

import argparse
import json
import os
import shutil
import subprocess
import sys
import tempfile
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Callable

__all__ = ["BACKENDS", "Probe", "REQUESTS", "RECORD_SCHEMA", "ResolvedSandboxBackend", "SandboxBackendError",
           "main", "probe_docker", "probe_udocker", "resolve_sandbox_backend"]

RECORD_SCHEMA = "thundersync-sandbox-backend-v1"
BACKENDS = ("docker", "udocker")
REQUESTS = ("auto", *BACKENDS)
DEFAULT_PROBE_TIMEOUT_S = 15.0
Runner = Callable[..., subprocess.CompletedProcess]


class SandboxBackendError(RuntimeError):
    pass


@dataclass(frozen=True, slots=True)
class Probe:
    usable: bool
    version: str | None
    detail: str

    def as_record(self) -> dict[str, Any]:
        return {"usable": self.usable, "version": self.version, "detail": self.detail}


@dataclass(frozen=True, slots=True)
class ResolvedSandboxBackend:
    requested: str
    backend: str
    decided_by: str
    docker: Probe | None
    udocker: Probe | None

    @property
    def version(self) -> str | None:
        p = self.docker if self.backend == "docker" else self.udocker
        return None if p is None else p.version

    def as_record(self) -> dict[str, Any]:
        return {"schema": RECORD_SCHEMA, "requested": self.requested, "backend": self.backend,
                "decided_by": self.decided_by, "version": self.version,
                "docker": None if self.docker is None else self.docker.as_record(),
                "udocker": None if self.udocker is None else self.udocker.as_record()}

    def factory(self):
        """The sandbox class of the resolved backend."""
        if self.backend == "docker":
            from thundersync_b200.rollout.docker_sandbox import DockerSandbox

            return DockerSandbox
        from thundersync_b200.rollout.udocker_sandbox import UDockerSandbox

        return UDockerSandbox


def _exe(path: str) -> str | None:
    found = shutil.which(path)
    if found:
        return found
    p = Path(path)
    return str(p) if p.is_file() and os.access(p, os.X_OK) else None


def _call(runner: Runner, argv: list[str], timeout_s: float, env=None):
    try:
        kw = {"capture_output": True, "text": True, "timeout": timeout_s}
        if env is not None:
            kw["env"] = env
        return runner(argv, **kw)
    except subprocess.TimeoutExpired:
        return f"`{' '.join(argv)}` did not answer within {timeout_s:g} s"
    except OSError as exc:
        return f"`{' '.join(argv)}` could not start: {exc}"


def _last_line(cp) -> str:
    lines = (cp.stderr or cp.stdout or "").strip().splitlines()
    return lines[-1][:300] if lines else "no output"


def probe_docker(bin_path: str = "docker", *, timeout_s: float = DEFAULT_PROBE_TIMEOUT_S,
                 runner: Runner = subprocess.run) -> Probe:
    """Usable iff ``docker version`` reports a *server* version (the daemon answers this user)."""
    exe = _exe(bin_path)
    if exe is None:
        return Probe(False, None, f"no {bin_path!r} executable on PATH")
    cp = _call(runner, [exe, "version", "--format", "{{.Server.Version}}"], timeout_s)
    if isinstance(cp, str):
        return Probe(False, None, cp)
    ver = cp.stdout.strip()
    if cp.returncode != 0 or not ver:
        return Probe(False, None, f"docker daemon unusable (exit {cp.returncode}): {_last_line(cp)}")
    return Probe(True, ver.splitlines()[-1], f"server {exe}")


def probe_udocker(bin_path: str = "udocker", *, timeout_s: float = DEFAULT_PROBE_TIMEOUT_S,
                  runner: Runner = subprocess.run) -> Probe:
    """Usable iff ``udocker version`` runs (against a throwaway UDOCKER_DIR, never the real store)."""
    exe = _exe(bin_path)
    if exe is None:
        return Probe(False, None, f"no udocker executable at {bin_path!r}")
    with tempfile.TemporaryDirectory(prefix="udocker-probe-") as scratch:
        cp = _call(runner, [exe, "version"], timeout_s, env={**os.environ, "UDOCKER_DIR": scratch})
    if isinstance(cp, str):
        return Probe(False, None, cp)
    if cp.returncode != 0:
        return Probe(False, None, f"udocker unusable (exit {cp.returncode}): {_last_line(cp)}")
    out = cp.stdout.strip()
    ver = next((ln.split(":", 1)[1].strip() for ln in out.splitlines() if ln.lower().startswith("version")),
               out.splitlines()[0] if out else "unknown")
    return Probe(True, ver, f"executable {exe}")


def resolve_sandbox_backend(requested: str, *, docker_bin: str | None = None, udocker_bin: str | None = None,
                            timeout_s: float = DEFAULT_PROBE_TIMEOUT_S,
                            runner: Runner = subprocess.run) -> ResolvedSandboxBackend:
    if requested not in REQUESTS:
        raise SandboxBackendError(f"sandbox backend {requested!r} is not one of {', '.join(REQUESTS)}")
    dbin = docker_bin or os.environ.get("THUNDERSYNC_DOCKER_BIN", "docker")
    ubin = udocker_bin or os.environ.get("THUNDERSYNC_UDOCKER_BIN", "udocker")
    if requested == "docker":
        d = probe_docker(dbin, timeout_s=timeout_s, runner=runner)
        if not d.usable:
            raise SandboxBackendError(f"sandbox backend docker was requested and is not usable: {d.detail}")
        return ResolvedSandboxBackend(requested, "docker", "explicit_request", d, None)
    if requested == "udocker":
        u = probe_udocker(ubin, timeout_s=timeout_s, runner=runner)
        if not u.usable:
            raise SandboxBackendError(f"sandbox backend udocker was requested and is not usable: {u.detail}")
        return ResolvedSandboxBackend(requested, "udocker", "explicit_request", None, u)
    d = probe_docker(dbin, timeout_s=timeout_s, runner=runner)
    if d.usable:
        return ResolvedSandboxBackend(requested, "docker", "auto_docker_daemon_usable", d, None)
    u = probe_udocker(ubin, timeout_s=timeout_s, runner=runner)
    if u.usable:
        return ResolvedSandboxBackend(requested, "udocker", "auto_docker_unusable_udocker_available", d, u)
    raise SandboxBackendError(f"no sandbox backend is usable: docker: {d.detail}; udocker: {u.detail}")


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--requested", choices=REQUESTS, required=True)
    ap.add_argument("--docker-bin", default=None)
    ap.add_argument("--udocker-bin", default=None)
    ap.add_argument("--timeout-s", type=float, default=DEFAULT_PROBE_TIMEOUT_S)
    args = ap.parse_args(argv)
    try:
        r = resolve_sandbox_backend(args.requested, docker_bin=args.docker_bin, udocker_bin=args.udocker_bin,
                                    timeout_s=args.timeout_s)
    except SandboxBackendError as exc:
        print(f"sandbox backend: {exc}", file=sys.stderr)
        return 2
    print(json.dumps(r.as_record(), sort_keys=True))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
