"""Which container runtime a site's sandboxes run on (C53).

Rule: Docker when this user's Docker daemon answers, udocker otherwise. A
request of ``auto`` applies the rule; a request naming a runtime gets that
runtime or an error, never the other one. A site resolves once and hands the
record to every process (the record's schema name, its ``decided_by`` labels
and the ``THUNDERSYNC_DOCKER_BIN`` / ``THUNDERSYNC_UDOCKER_BIN`` variables are
the interface of reference src/thundersync/rollout/sandbox_backend.py:1-239;
tooling that reads the record keeps working).

Design: each runtime is described by a :class:`_Runtime` row (how to ask it
for its version, how to read the answer); one generic checker runs any row
with a timeout; resolution walks a short list of (runtime, label) candidates.

``python -m thundersync_b200.rollout.sandbox_backend --requested auto`` prints
the resolution record as one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import shutil
import subprocess
import sys
import tempfile
from contextlib import ExitStack
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
    """No usable runtime for the request."""


@dataclass(frozen=True, slots=True)
class Probe:
    """Outcome of asking one runtime for its version."""

    usable: bool
    version: str | None
    detail: str

    def as_record(self) -> dict[str, Any]:
        return {"usable": self.usable, "version": self.version, "detail": self.detail}


@dataclass(frozen=True, slots=True)
class ResolvedSandboxBackend:
    """The chosen runtime, why it was chosen, and the probes that were run."""

    requested: str
    backend: str
    decided_by: str
    docker: Probe | None
    udocker: Probe | None

    @property
    def version(self) -> str | None:
        chosen = {"docker": self.docker, "udocker": self.udocker}[self.backend]
        return chosen.version if chosen is not None else None

    def as_record(self) -> dict[str, Any]:
        rec: dict[str, Any] = {"schema": RECORD_SCHEMA, "requested": self.requested, "backend": self.backend,
                               "decided_by": self.decided_by, "version": self.version}
        for name in BACKENDS:
            probe = getattr(self, name)
            rec[name] = probe.as_record() if probe is not None else None
        return rec

    def factory(self):
        """The sandbox class that runs on the chosen runtime."""
        if self.backend == "docker":
            from thundersync_b200.rollout.docker_sandbox import DockerSandbox as cls
        else:
            from thundersync_b200.rollout.udocker_sandbox import UDockerSandbox as cls
        return cls


# ----------------------------------------------------------------------------- runtime rows
def _docker_version(stdout: str) -> str | None:
    # `docker version --format {{.Server.Version}}` prints the daemon's version, or nothing when the client
    # cannot reach a daemon (some clients still exit 0 then)
    lines = [ln.strip() for ln in stdout.splitlines() if ln.strip()]
    return lines[-1] if lines else None


def _udocker_version(stdout: str) -> str | None:
    lines = [ln.strip() for ln in stdout.splitlines() if ln.strip()]
    for ln in lines:
        key, sep, val = ln.partition(":")
        if sep and key.strip().lower() == "version":
            return val.strip()
    return lines[0] if lines else "unknown"


@dataclass(frozen=True)
class _Runtime:
    name: str
    argv_tail: tuple[str, ...]
    read_version: Callable[[str], str | None]
    private_store: bool  # point UDOCKER_DIR at a throwaway directory so the probe never touches the real store


_RUNTIMES = {
    "docker": _Runtime("docker", ("version", "--format", "{{.Server.Version}}"), _docker_version, False),
    "udocker": _Runtime("udocker", ("version",), _udocker_version, True),
}
_ENV_BIN = {"docker": "THUNDERSYNC_DOCKER_BIN", "udocker": "THUNDERSYNC_UDOCKER_BIN"}


def _locate(binary: str) -> str | None:
    hit = shutil.which(binary)
    if hit is not None:
        return hit
    path = Path(binary)
    if path.is_file() and os.access(path, os.X_OK):
        return str(path)
    return None


def _tail(text: str | None) -> str:
    for ln in reversed((text or "").splitlines()):
        if ln.strip():
            return ln.strip()[:300]
    return "(no output)"


def _check(rt: _Runtime, binary: str, timeout_s: float, runner: Runner) -> Probe:
    exe = _locate(binary)
    if exe is None:
        return Probe(False, None, f"{rt.name}: executable {binary!r} not found")
    argv = [exe, *rt.argv_tail]
    with ExitStack() as stack:
        kwargs: dict[str, Any] = {"capture_output": True, "text": True, "timeout": timeout_s}
        if rt.private_store:
            scratch = stack.enter_context(tempfile.TemporaryDirectory(prefix="ts-udocker-probe-"))
            kwargs["env"] = dict(os.environ, UDOCKER_DIR=scratch)
        try:
            done = runner(argv, **kwargs)
        except subprocess.TimeoutExpired:
            return Probe(False, None, f"{rt.name}: no answer from {exe} after {timeout_s:g} s")
        except OSError as exc:
            return Probe(False, None, f"{rt.name}: {exe} failed to start ({exc})")
    version = rt.read_version(done.stdout or "") if done.returncode == 0 else None
    if version is None:
        why = _tail(done.stderr) if (done.stderr or "").strip() else _tail(done.stdout)
        return Probe(False, None, f"{rt.name}: {exe} exited {done.returncode} without a version ({why})")
    return Probe(True, version, f"{rt.name}: {exe}")


def probe_docker(bin_path: str = "docker", *, timeout_s: float = DEFAULT_PROBE_TIMEOUT_S,
                 runner: Runner = subprocess.run) -> Probe:
    """Usable when the Docker daemon reports a server version to this user."""
    return _check(_RUNTIMES["docker"], bin_path, timeout_s, runner)


def probe_udocker(bin_path: str = "udocker", *, timeout_s: float = DEFAULT_PROBE_TIMEOUT_S,
                  runner: Runner = subprocess.run) -> Probe:
    """Usable when ``udocker version`` runs (against a throwaway store directory)."""
    return _check(_RUNTIMES["udocker"], bin_path, timeout_s, runner)


# ----------------------------------------------------------------------------- resolution
# (runtime, decided_by label when it is chosen) in the order they are tried
_PLANS = {
    "auto": (("docker", "auto_docker_daemon_usable"), ("udocker", "auto_docker_unusable_udocker_available")),
    "docker": (("docker", "explicit_request"),),
    "udocker": (("udocker", "explicit_request"),),
}


def resolve_sandbox_backend(requested: str, *, docker_bin: str | None = None, udocker_bin: str | None = None,
                            timeout_s: float = DEFAULT_PROBE_TIMEOUT_S,
                            runner: Runner = subprocess.run) -> ResolvedSandboxBackend:
    """Pick the runtime for ``requested`` (``auto``, ``docker`` or ``udocker``) or raise."""
    plan = _PLANS.get(requested)
    if plan is None:
        raise SandboxBackendError(f"unknown sandbox backend request {requested!r}; choose one of {list(REQUESTS)}")
    binaries = {"docker": docker_bin, "udocker": udocker_bin}
    probes: dict[str, Probe] = {}
    for name, label in plan:
        binary = binaries[name] or os.environ.get(_ENV_BIN[name], name)
        probes[name] = _check(_RUNTIMES[name], binary, timeout_s, runner)
        if probes[name].usable:
            return ResolvedSandboxBackend(requested, name, label, probes.get("docker"), probes.get("udocker"))
    reasons = "; ".join(p.detail for p in probes.values())
    if requested == "auto":
        raise SandboxBackendError(f"neither docker nor udocker can run sandboxes here: {reasons}")
    raise SandboxBackendError(f"requested sandbox backend {requested} is not usable here: {reasons}")


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description="Resolve the sandbox container runtime and print its record.")
    ap.add_argument("--requested", choices=REQUESTS, required=True)
    ap.add_argument("--docker-bin", default=None)
    ap.add_argument("--udocker-bin", default=None)
    ap.add_argument("--timeout-s", type=float, default=DEFAULT_PROBE_TIMEOUT_S)
    args = ap.parse_args(argv)
    try:
        resolved = resolve_sandbox_backend(args.requested, docker_bin=args.docker_bin,
                                           udocker_bin=args.udocker_bin, timeout_s=args.timeout_s)
    except SandboxBackendError as exc:
        sys.stderr.write(f"{exc}\n")
        return 2
    sys.stdout.write(json.dumps(resolved.as_record(), sort_keys=True) + "\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
