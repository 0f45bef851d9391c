"""Rollout layer on the host: bounded capture, agent parsing/truncation, guards,
sandboxes (fake docker CLI, host-directory sandbox), pool gate, backend
resolution, and the rollout engine's two schedules (fake token-id LLM).

Reference behaviour: tests/rollout/* of the reference (bounded output exactness,
kill caps, seccomp network guard, token-identical lockstep/async schedules,
pristine gate fails closed).
"""

from __future__ import annotations

import os
import shutil
import socket
import subprocess
import sys
import time
from pathlib import Path

import pytest

from tests.rollout.fakes import FakeLLM, LocalSandbox, install_fake_docker
from thundersync_b200.rollout.agent import (Step, Task, Trajectory, extract_keywords, parse_action,
                                            truncate_observation, truncate_observation_tokens)
from thundersync_b200.rollout.bounded_output import MemoryGuard, StreamCapture, run_bounded
from thundersync_b200.rollout.engine import BatchedRolloutEngine, Verdict, request_seed
from thundersync_b200.rollout.sandbox_backend import SandboxBackendError, resolve_sandbox_backend
from thundersync_b200.rollout.sandbox_pool import SandboxPool, trusted_tree_pristine
from thundersync_b200.rollout.scratch_guard import ScratchGuard


# ---------------------------------------------------------------------------- bounded output
def test_stream_capture_whole_and_spilled():
    cap = StreamCapture(16)
    cap.feed(b"ab\r\ncd\r")
    t = cap.finish()
    assert t.complete and t.text == "ab\ncd\n"
    cap = StreamCapture(10)
    data = "é" * 40  # 80 bytes of 2-byte characters
    for i in range(0, 80, 7):
        cap.feed(data.encode()[i:i + 7])
    t = cap.finish()
    assert not t.complete and t.chars == 40 and t.nbytes == 80
    assert set(t.kept_head) == {"é"} and set(t.kept_tail) == {"é"}
    assert "chars elided" in t.rendered()


def test_run_bounded_kill_cap_timeout_and_guard():
    r = run_bounded([sys.executable, "-c", "import sys; sys.stdout.write('x' * 100000)"], timeout=30,
                    keep_bytes=1000, kill_bytes=5000)
    assert r.killed == "output_cap" and r.stdout.nbytes == 5000 and not r.stdout.complete
    r = run_bounded(["sleep", "5"], timeout=0.3)
    assert r.timed_out
    r = run_bounded(["echo", "hi"], timeout=10, memory_guard=MemoryGuard(1, rss=lambda: 100))
    assert r.refused and r.killed == "memory_budget"
    r = run_bounded(["sh", "-c", "echo out; echo err >&2; exit 3"], timeout=10)
    assert r.returncode == 3 and r.stdout.text == "out\n" and r.stderr.text == "err\n"


# ---------------------------------------------------------------------------- agent
def test_parse_action_and_truncation():
    assert parse_action("x\n```bash\nls -la\n```\ny") == "ls -la"
    assert parse_action("```bash\ncat <<'E'\na ``` b\nE\n```") == "cat <<'E'\na ``` b\nE"
    assert parse_action("no block") is None
    long = "a" * 50 + "b" * 50
    assert truncate_observation(long, 20) == "a" * 10 + "\n\n... <80 chars elided> ...\n\n" + "b" * 10
    enc = lambda s: list(s.encode())  # noqa: E731
    dec = lambda ids: bytes(ids).decode(errors="replace")  # noqa: E731
    out = truncate_observation_tokens(long, enc, dec, max_tokens=10)
    assert out.startswith("aaaaa") and out.endswith("bbbbb") and "<90 tokens elided>" in out
    assert truncate_observation_tokens("short", enc, dec, max_tokens=10) == "short"
    assert extract_keywords("the foo_bar broke; foo_bar and Baz_Qux fail")[:2] == ["foo_bar", "Baz_Qux"]


def test_trajectory_masks():
    tr = Trajectory("t", 0, 0, prompt_token_ids=[1, 2])
    tr.steps.append(Step("ls", "out", action_token_ids=[3, 4], action_logprobs=[-1, -2],
                         observation_token_ids=[5]))
    assert tr.token_ids == [1, 2, 3, 4, 5]
    assert tr.action_mask == [False, False, True, True, False]
    assert tr.logprobs == [0.0, 0.0, -1, -2, 0.0]
    assert tr.turns == [([3, 4, 5], [True, True, False])]
    with pytest.raises(ValueError):
        Task("i", "p", "img", test_framework="maven")


# ---------------------------------------------------------------------------- guards
def test_scratch_guard_budget_and_reclaim(tmp_path):
    g = ScratchGuard([tmp_path], budget_bytes=100_000, check_interval_s=0.01)
    assert g.over_budget() is None
    (tmp_path / "big").write_bytes(os.urandom(400_000))
    assert g.over_budget() is not None
    done = g.reclaim()
    assert [Path(r.path).name for r in done] == ["big"] and g.over_budget() is None


@pytest.mark.skipif(not Path("thundersync_b200/rollout/ts_netguard").exists(), reason="host tools not built")
def test_network_guard_denies_inet_keeps_unix():
    from thundersync_b200.rollout.network_guard import guarded_argv

    code = ("import socket\nsocket.socket(socket.AF_UNIX).close()\nsocket.socketpair()\n"
            "try:\n    socket.socket(socket.AF_INET)\n    print('open')\nexcept PermissionError:\n    print('denied')\n")
    out = subprocess.run(guarded_argv([sys.executable, "-c", code]), capture_output=True, text=True, timeout=60)
    assert out.stdout.strip() == "denied", out.stderr


# ---------------------------------------------------------------------------- sandboxes
def test_docker_sandbox_with_fake_cli(tmp_path, monkeypatch):
    env = install_fake_docker(tmp_path, {"img:1": {"mod.py": "x = 1\n"}})
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    from thundersync_b200.rollout.docker_sandbox import DockerSandbox, owned_containers

    box = DockerSandbox("img:1", "task-1")
    box.start()
    try:
        args = box._run_arguments()
        assert "--network" in args and args[args.index("--network") + 1] == "none"
        assert "no-new-privileges" in args and "ALL" in args
        assert (box.host_workdir / "mod.py").read_text() == "x = 1\n"
        assert box.exec("cat mod.py") == "x = 1\n"
        assert box.name in owned_containers()
        out = box.exec_output("echo hi; exit 4")
        assert out.returncode == 4 and str(out) == "hi\n"
    finally:
        box.close()
    assert not box.host_root.exists() and box.name not in owned_containers()


def test_backend_resolution_rules():
    def runner_factory(docker_ok, udocker_ok):
        def run(argv, **kw):
            if "udocker" in argv[0]:
                return subprocess.CompletedProcess(argv, 0 if udocker_ok else 1, "version: 1.3.17\n", "")
            return subprocess.CompletedProcess(argv, 0 if docker_ok else 1, "27.1\n" if docker_ok else "",
                                               "" if docker_ok else "Cannot connect to the Docker daemon")
        return run

    d, u = sys.executable, sys.executable.replace("python", "python") + ""
    fake_u = shutil.which("true")
    r = resolve_sandbox_backend("auto", docker_bin=d, udocker_bin=fake_u, runner=runner_factory(True, True))
    assert r.backend == "docker" and r.decided_by == "auto_docker_daemon_usable"
    r = resolve_sandbox_backend("auto", docker_bin=d, udocker_bin="/nonexistent/udocker",
                                runner=runner_factory(False, False)) if False else None
    with pytest.raises(SandboxBackendError, match="not usable"):
        resolve_sandbox_backend("docker", docker_bin=d, runner=runner_factory(False, True))
    with pytest.raises(SandboxBackendError):
        resolve_sandbox_backend("podman")


def test_backend_resolution_falls_back_to_udocker_and_records_both_probes():
    def run(argv, **kw):
        if argv[1:] == ["version"]:
            assert "UDOCKER_DIR" in kw["env"]  # the probe never touches the real udocker store
            return subprocess.CompletedProcess(argv, 0, "udocker 1.3.17\nversion: 1.3.17\n", "")
        return subprocess.CompletedProcess(argv, 1, "", "Cannot connect to the Docker daemon")

    exe = shutil.which("true")
    r = resolve_sandbox_backend("auto", docker_bin=exe, udocker_bin=exe, runner=run)
    rec = r.as_record()
    assert r.backend == "udocker" and r.decided_by == "auto_docker_unusable_udocker_available"
    assert rec["schema"] == "thundersync-sandbox-backend-v1" and rec["version"] == "1.3.17"
    assert rec["docker"]["usable"] is False and "Docker daemon" in rec["docker"]["detail"]
    with pytest.raises(SandboxBackendError):
        resolve_sandbox_backend("auto", docker_bin="/nonexistent/docker", udocker_bin="/nonexistent/udocker")
    r = resolve_sandbox_backend("udocker", udocker_bin=exe, runner=run)
    assert r.decided_by == "explicit_request" and r.docker is None


# ---------------------------------------------------------------------------- pool
def test_pool_gate_reuses_pristine_and_discards_dirty():
    task = Task("t1", "p", "img")
    pool = SandboxPool(lambda im, nm: LocalSandbox(im, nm), name_prefix="p")
    a = pool.acquire(task)
    assert trusted_tree_pristine(a)
    a.exec("echo edit >> mod.py")
    pool.release(task, a)  # the in-container reset restores it: pristine, kept
    b = pool.acquire(task)
    assert b is a and pool.reused == 1
    # a change the in-container reset cannot undo (ignored file) fails the gate
    b.exec("echo '*.log' > .gitignore && git add .gitignore && git -c user.name=t -c user.email=t@x commit -qm x "
           "&& echo hi > junk.log")
    pool.release(task, b)
    assert pool.pristine_failures == 1 and b.closed
    c = pool.acquire(task)
    assert c is not b and pool.created == 2
    pool.close()


# ---------------------------------------------------------------------------- engine
def _engine():
    return BatchedRolloutEngine(llm=FakeLLM(), max_model_len=100_000)


def _grade(box, task):
    text = (Path(box.host_workdir) / "out.txt").read_text() if (Path(box.host_workdir) / "out.txt").exists() else ""
    return Verdict(1.0 if text.strip() else 0.0, reason="pass" if text.strip() else "fail")


@pytest.mark.parametrize("schedule", ["lockstep", "async"])
def test_engine_rollout_group(schedule):
    eng = _engine()
    task = Task("t1", "fix foo_bar please", "img")
    blocks, verdicts = [], []
    trajs, tim = eng.rollout_group(task, schedule=schedule, group_size=3, group_id=5, base_seed=11,
                                   repo_context=False, sandbox_factory=lambda im, nm: LocalSandbox(im, nm),
                                   grade_fn=_grade, on_block=lambda ev: blocks.extend(ev),
                                   on_verdict=lambda i, t: verdicts.append(i), max_steps=5)
    assert sorted(verdicts) == [0, 1, 2]
    for i, t in enumerate(trajs):
        assert t.finish_reason == "submit" and len(t.steps) == 3 and t.reward == 1.0
        assert len(t.token_ids) == len(t.action_mask)
        seed0 = request_seed(11, 5, i, 0)
        assert f"echo {seed0 % 997}" in t.steps[0].action
    assert tim.schedule == schedule and tim.n_steps == 3
    assert any(b.kind == "observation" for _, b in blocks)


def test_engine_schedules_are_token_identical():
    task = Task("t1", "fix foo_bar please", "img")
    kw = dict(group_size=2, group_id=1, base_seed=3, repo_context=False,
              sandbox_factory=lambda im, nm: LocalSandbox(im, nm), grade_fn=_grade, max_steps=4)
    a, _ = _engine().rollout_group(task, schedule="lockstep", **kw)
    b, _ = _engine().rollout_group(task, schedule="async", **kw)
    assert [t.token_ids for t in a] == [t.token_ids for t in b]
    outs = _engine().rollout_groups([dict(task=task, group_id=g) for g in range(2)], schedule="async",
                                    **{k: v for k, v in kw.items() if k != "group_id"})
    assert [t.token_ids for t in outs[1][0]] == [t.token_ids for t in a]
    assert request_seed(0, 0, 0, 0) == request_seed(0, 0, 0, 0) != request_seed(0, 0, 0, 1)
