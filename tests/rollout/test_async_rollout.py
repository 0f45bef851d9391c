"""The rollout engine's two schedules: what changes is when work runs, never what is sampled.

Reference behaviour: tests/rollout/test_async_rollout.py of the reference (makespan, callback order,
token identity across schedules, verdict timing, batched generation, bounded failure). Rollouts run on a
deterministic token-id fake LLM and host-directory sandboxes whose tool latency differs per rollout.
"""

from __future__ import annotations

import threading
import time
from pathlib import Path

import pytest

from tests.rollout.fakes import FakeLLM, LocalSandbox
from thundersync_b200.rollout.agent import Task
from thundersync_b200.rollout.engine import BatchedRolloutEngine, Verdict, request_seed

DELAYS = [0.30, 0.02, 0.02, 0.02]  # rollout 0's tool calls are slow, the others fast


class SlowSandbox(LocalSandbox):
    def __init__(self, image, name, **kw):
        super().__init__(image, name, **kw)
        self.delay = DELAYS[int(name.rsplit("-", 1)[1])]

    def exec_output(self, command, **kw):
        if "out.txt" in command:
            time.sleep(self.delay)
        return super().exec_output(command, **kw)


def _grade(box, task):
    text = (Path(box.host_workdir) / "out.txt").read_text() if (Path(box.host_workdir) / "out.txt").exists() else ""
    return Verdict(1.0 if text.strip() else 0.0, reason="pass" if text.strip() else "fail")


def _run(schedule, llm=None, **kw):
    eng = BatchedRolloutEngine(llm=llm or FakeLLM(), max_model_len=100_000)
    events = {"blocks": [], "verdicts": [], "completed": [], "concurrent": 0}
    busy = threading.Lock()

    def on_block(ev):
        if not busy.acquire(blocking=False):  # trainer callbacks must never overlap
            events["concurrent"] += 1
            return
        try:
            events["blocks"].extend(ev)
            time.sleep(0.001)
        finally:
            busy.release()

    t0 = time.perf_counter()
    trajs, tim = eng.rollout_group(
        Task("t1", "fix foo_bar please", "img"), schedule=schedule, group_size=len(DELAYS), group_id=3,
        base_seed=7, repo_context=False, sandbox_factory=lambda im, nm: SlowSandbox(im, nm), grade_fn=_grade,
        on_block=on_block, on_verdict=lambda i, t: events["verdicts"].append((i, time.perf_counter())),
        on_trajectory_complete=lambda i, t: events["completed"].append((i, time.perf_counter())),
        max_steps=6, **kw)
    events["wall"] = time.perf_counter() - t0
    return trajs, tim, events, eng


def test_async_makespan_beats_lockstep_under_heterogeneous_tool_latency():
    _, _, lock_ev, _ = _run("lockstep")
    _, _, async_ev, _ = _run("async")
    # lockstep pays the slowest rollout's tool latency at every round barrier; async lets the fast rollouts
    # finish while the slow one is still running, so the fast ones' verdicts come early
    first_async = min(t for _, t in async_ev["verdicts"])
    last_async = max(t for _, t in async_ev["verdicts"])
    assert last_async - first_async > 0.2
    lock_times = [t for _, t in lock_ev["verdicts"]]
    assert max(lock_times) - min(lock_times) < 0.2  # lockstep grades everyone together at the end


def test_trajectories_are_token_identical_across_schedules():
    a, _, _, _ = _run("lockstep")
    b, _, _, _ = _run("async")
    for x, y in zip(a, b):
        assert x.token_ids == y.token_ids and x.action_mask == y.action_mask
        assert x.finish_reason == y.finish_reason and x.reward == y.reward
        assert [s.action for s in x.steps] == [s.action for s in y.steps]


def test_each_turn_samples_with_its_own_request_seed():
    trajs, _, _, _ = _run("async")
    for i, t in enumerate(trajs):
        for k, step in enumerate(t.steps[:2]):
            assert f"echo {request_seed(7, 3, i, k) % 997}" in step.action


def test_trainer_callbacks_are_serialised_and_ordered_per_trajectory():
    _, _, ev, _ = _run("async")
    assert ev["concurrent"] == 0
    per_traj: dict[int, list] = {}
    for i, block in ev["blocks"]:
        per_traj.setdefault(i, []).append(block)
    assert sorted(per_traj) == [0, 1, 2, 3]
    done = dict(ev["completed"])
    for i, t in ev["verdicts"]:
        assert done[i] <= t  # a trajectory completes before its verdict fires


def test_generation_stays_batched_without_the_round_barrier():
    llm = FakeLLM()
    _run("async", llm=llm)
    assert max(llm.calls) > 1  # concurrent requests are served in one generate call


def test_unknown_schedule_and_oversized_prompt_are_refused():
    eng = BatchedRolloutEngine(llm=FakeLLM(), max_model_len=100_000)
    with pytest.raises(ValueError, match="schedule"):
        eng.rollout_group(Task("t", "p", "img"), schedule="eager", group_size=1)
    with pytest.raises(ValueError, match="max_prompt_tokens"):
        eng.rollout_group(Task("t", "p", "img"), schedule="async", group_size=1, max_prompt_tokens=0)
    with pytest.raises(ValueError, match="over max_prompt_tokens"):
        eng.rollout_group(Task("t", "x" * 200, "img"), schedule="async", group_size=1, repo_context=False,
                          max_prompt_tokens=16, sandbox_factory=lambda im, nm: LocalSandbox(im, nm))


class FailingLLM(FakeLLM):
    def generate_token_ids(self, prompts, caps, temperature, top_p, seeds):
        raise RuntimeError("generation backend died")


@pytest.mark.parametrize("schedule", ["lockstep", "async"])
def test_generation_failure_reaches_the_caller_instead_of_hanging(schedule):
    t0 = time.perf_counter()
    with pytest.raises(RuntimeError, match="generation backend died"):
        _run(schedule, llm=FailingLLM())
    assert time.perf_counter() - t0 < 30
