"""Batched rollout engine over vLLM's offline API, with trusted grading (C45).

Generation goes through vLLM's offline ``LLM.generate`` on token-id prompts,
so the trainer receives the exact generated token ids (re-encoding strings
could shift token boundaries and invent divergence). Two schedules:

* ``lockstep`` — every live rollout generates one action (one batched
  ``generate``), then all tools run, then the next round; grading happens at
  a group barrier;
* ``async`` — one worker thread per rollout owns its turn loop and submits to
  a :class:`_GenerationBroker`, which coalesces whatever requests are
  outstanding into one ``generate`` call; each trajectory is graded at its
  own finish and ``on_verdict`` fires per trajectory; ``rollout_groups`` runs
  several groups against one broker.

The schedule changes *when* work runs, not *what* is sampled: every request
carries its own seed, :func:`request_seed` ``(base_seed, group, rollout,
turn)``, and vLLM seeds each sequence independently, so the returned ids are
a function of (prompt ids, seed) alone.

Grading (:func:`grade`) runs FAIL_TO_PASS (and PASS_TO_PASS for regressions)
with structured reports — pytest JUnit XML per selector batch, or one ``go
test -json`` — and returns a :class:`Verdict` that never hides a missing
test behind a float. :func:`grade_isolated` grades the policy's repository
patch (captured on the host against the trusted sealed tree) in a fresh
verifier sandbox (reference: src/thundersync/rollout/engine.py:1-2460).
"""

from __future__ import annotations

import hashlib
import json
import logging
import os
import queue
import secrets
import shlex
import struct
import subprocess
import threading
import time
import xml.etree.ElementTree as ET
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Callable, Sequence

from thundersync_b200.rollout.agent import (CONTEXT_TEMPLATE, SYSTEM_PROMPT, TASK_TEMPLATE, Step, Task, Trajectory,
                                            build_repo_context, parse_action, truncate_observation_tokens)
from thundersync_b200.rollout.bounded_output import command_output, run_bounded

log = logging.getLogger(__name__)

__all__ = [
    "BatchTimings", "BatchedRolloutEngine", "COUPLED_ROLLOUT_SLOT", "CommittedBlock", "GenResult",
    "HOST_GIT_CONFIG", "HOST_GIT_ENV", "PARSE_ERROR_OBSERVATION", "PolicyPatchRejected", "Verdict",
    "capture_policy_patch", "capture_trusted_bug_tree", "grade", "grade_isolated", "new_sandbox", "parse_test_ids",
    "request_seed", "run_tests",
]

PARSE_ERROR_OBSERVATION = "No command found. Reply with exactly one ```bash ... ``` block."
REPORT_KEEP_BYTES = 64 << 20
COUPLED_ROLLOUT_SLOT = 0
HOST_GIT_CONFIG = ["-c", "core.autocrlf=false", "-c", "core.fileMode=true", "-c", "safe.directory=*",
                   "-c", "user.name=thundersync", "-c", "user.email=thundersync@localhost"]
HOST_GIT_ENV = {"GIT_CONFIG_NOSYSTEM": "1", "GIT_TERMINAL_PROMPT": "0", "GIT_NO_REPLACE_OBJECTS": "1"}
RUNTIME_EXCLUDES = [":(exclude).git", ":(exclude,glob).git/**", ":(exclude,glob)**/__pycache__/**",
                    ":(exclude,glob)**/*.pyc", ":(exclude,glob)**/*.pyo", ":(exclude,glob)**/*.egg-info/**",
                    ":(exclude,glob)**/.pytest_cache/**"]


@dataclass
class GenResult:
    token_ids: list[int]
    logprobs: list[float]
    text: str
    finish_reason: str = ""
    ready_at: float | None = None


@dataclass(frozen=True)
class CommittedBlock:
    """An immutable piece of a trajectory as it is emitted: an action (opener + generated) or an observation."""
    step_index: int
    kind: str
    token_ids: tuple[int, ...]
    scored: tuple[bool, ...]
    committed_at: float
    terminal_reason_at_commit: str | None = None

    def __post_init__(self) -> None:
        if self.kind not in ("action", "observation"):
            raise ValueError(f"unknown block kind {self.kind!r}")
        if len(self.token_ids) != len(self.scored):
            raise ValueError("token_ids and scored differ in length")


@dataclass
class BatchTimings:
    generation_s: float = 0.0
    generation_batch_sizes: list[int] = field(default_factory=list)
    shared_generation_s: float = 0.0
    shared_generation_batch_sizes: list[int] = field(default_factory=list)
    shared_generation_prompt_tokens: int = 0
    shared_generation_completion_tokens: int = 0
    tool_s: float = 0.0
    verify_s: float = 0.0
    graded_at: float = 0.0
    schedule: str = "lockstep"
    rollout_wall_s: float = 0.0
    verdict_at: list[float] = field(default_factory=list)
    trajectory_completed_at: list[float] = field(default_factory=list)
    n_steps: int = 0
    tool_calls: int = 0
    model_rows: int = 0
    logical_rows: int = 0

    @property
    def compression(self) -> float:
        return self.logical_rows / max(self.model_rows, 1)


def parse_test_ids(ids) -> list[str]:
    if isinstance(ids, str):
        try:
            dec = json.loads(ids)
        except json.JSONDecodeError as exc:
            raise ValueError(f"test IDs must be a sequence or a JSON list, got {ids[:200]!r}") from exc
        if not isinstance(dec, list):
            raise ValueError(f"test IDs must decode to a JSON list, got {type(dec).__name__}")
        return [str(x) for x in dec]
    return list(ids or [])


@dataclass
class Verdict:
    reward: float
    passed: list[str] = field(default_factory=list)
    failed: list[str] = field(default_factory=list)
    missing: list[str] = field(default_factory=list)
    regressed: list[str] = field(default_factory=list)
    n_pass_to_pass: int = 0
    reason: str = ""

    @property
    def conclusive(self) -> bool:
        return not self.missing and self.reason not in ("timeout", "no_report")


class PolicyPatchRejected(RuntimeError):
    """The policy worktree cannot be represented as a bounded repository patch."""


def request_seed(base_seed: int, group_id: int, rollout_id: int, turn: int) -> int:
    """Non-negative 63-bit sampling seed: BLAKE2b-64 of the four signed 64-bit integers, shifted right by one.

    Stable across processes, Python versions and schedules; kept identical to
    the reference's definition so a seed names the same sample in both.
    """
    digest = hashlib.blake2b(struct.pack("<4q", base_seed, group_id, rollout_id, turn), digest_size=8).digest()
    return int.from_bytes(digest, "little") >> 1


def new_sandbox(factory: Callable[[str, str], Any], task: Task, name: str):
    box = factory(task.image_name, name)
    if task.requires_network:
        box.requires_network = True
    return box


# ---------------------------------------------------------------------------- trusted host-side git
def _git(args: list[str], **kw) -> subprocess.CompletedProcess:
    return subprocess.run(["git", *HOST_GIT_CONFIG, *args], capture_output=True, text=True,
                          env={**os.environ, **HOST_GIT_ENV}, timeout=kw.pop("timeout", 300), **kw)


def capture_trusted_bug_tree(sandbox: Any, rev: str = "HEAD") -> str:
    """Snapshot the sealed worktree into a host-owned bare store before any policy command runs.

    The tree id and store path are kept on the sandbox; the pristine gate and
    patch capture compare against them, never against the container's own
    (policy-writable) git state.
    """
    work = Path(sandbox.host_workdir)
    store = Path(getattr(sandbox, "host_root", work.parent)) / "trusted.git"
    if not store.exists():
        r = _git(["init", "-q", "--bare", str(store)])
        if r.returncode != 0:
            raise RuntimeError(f"trusted store init failed: {r.stderr}")
    base = [f"--git-dir={store}", f"--work-tree={work}"]
    for args in (["add", "-A", "--", ".", *RUNTIME_EXCLUDES],):
        r = _git([*base, *args])
        if r.returncode != 0:
            raise RuntimeError(f"trusted snapshot failed: {r.stderr}")
    tree = _git([*base, "write-tree"]).stdout.strip()
    if not tree:
        raise RuntimeError("trusted snapshot produced no tree")
    sandbox._thundersync_trusted_git_dir = str(store)
    sandbox._thundersync_trusted_tree = tree
    sandbox._thundersync_trusted_rev = rev
    return tree


def capture_policy_patch(sandbox: Any, *, max_bytes: int = 8 << 20) -> bytes:
    """The worktree's changes against the trusted sealed tree, as a binary git diff (host git only)."""
    store = getattr(sandbox, "_thundersync_trusted_git_dir", None)
    tree = getattr(sandbox, "_thundersync_trusted_tree", None)
    if store is None or tree is None:
        raise PolicyPatchRejected("no trusted tree was captured for this sandbox")
    base = ["git", *HOST_GIT_CONFIG, f"--git-dir={store}", f"--work-tree={sandbox.host_workdir}"]
    env = {**os.environ, **HOST_GIT_ENV}
    r = _git([f"--git-dir={store}", f"--work-tree={sandbox.host_workdir}", "add", "-A", "--", ".",
              *RUNTIME_EXCLUDES])
    if r.returncode != 0:
        raise PolicyPatchRejected(f"staging the policy worktree failed: {r.stderr[-400:]}")
    run = run_bounded([*base, "diff", "--cached", "--binary", tree], timeout=300, env=env, keep_bytes=max_bytes,
                      kill_bytes=max_bytes + (1 << 20))
    if run.timed_out or run.killed is not None or run.returncode != 0 or run.stdout.raw is None:
        raise PolicyPatchRejected(f"the policy patch exceeds {max_bytes} bytes or could not be captured")
    return run.stdout.raw


def source_diff(sandbox: Any) -> str:
    try:
        return capture_policy_patch(sandbox).decode("utf-8", errors="replace")
    except PolicyPatchRejected as exc:
        return f"<diff unavailable: {exc}>"


# ---------------------------------------------------------------------------- grading
def _read_report(sandbox: Any, path: str) -> str | None:
    out = command_output(sandbox, f"cat {path} 2>/dev/null", keep_bytes=REPORT_KEEP_BYTES)
    if not out.complete or out.killed is not None:
        log.warning("verifier report %s not read whole", path)
        return None
    return out.text


def _parse_junit(xml: str | None) -> ET.Element | None:
    """The report's root element, or None when it is empty, malformed, or declares a document type or
    entities (a report is written inside the policy's sandbox; entity expansion is never needed to read
    one and is refused rather than trusted)."""
    if not xml or not xml.strip():
        return None
    head = xml.upper()
    if "<!DOCTYPE" in head or "<!ENTITY" in head:
        return None
    try:
        return ET.fromstring(xml)
    except ET.ParseError:
        return None


def _junit_outcomes(root: ET.Element) -> dict[str, bool]:
    """{test id: passed} from a pytest JUnit report (ids as ``path::Class::name`` and ``classname.name``)."""
    out: dict[str, bool] = {}
    for case in root.iter("testcase"):
        bad = any(child.tag in ("failure", "error") for child in case)
        skipped = any(child.tag == "skipped" for child in case)
        name = case.get("name", "")
        cls = case.get("classname", "")
        keys = {f"{cls}.{name}" if cls else name, name}
        parts = cls.split(".")
        for cut in range(1, len(parts) + 1):
            mod = "/".join(parts[:cut]) + ".py"
            rest = parts[cut:]
            keys.add("::".join([mod, *rest, name]))
        for k in keys:
            if k in out and out[k] is False:
                continue
            out[k] = not bad and not skipped
    return out


def _selector_batches(ids: list[str], max_chars: int = 60000) -> list[list[str]]:
    batches, cur, size = [], [], 0
    for t in ids:
        if cur and size + len(t) + 3 > max_chars:
            batches.append(cur)
            cur, size = [], 0
        cur.append(t)
        size += len(t) + 3
    if cur:
        batches.append(cur)
    return batches


def _run_pytest(sandbox: Any, ids: list[str], timeout: float) -> tuple[dict[str, bool] | None, str]:
    results: dict[str, bool] = {}
    grade_token = secrets.token_hex(6)  # a fresh report path per grade: never read an earlier grade's report
    for k, batch in enumerate(_selector_batches(ids)):
        report = f"/tmp/ts-junit-{grade_token}-{k}.xml"
        sel = " ".join(shlex.quote(t) for t in batch)
        out = command_output(sandbox, f"rm -f {report}; python -m pytest -p no:cacheprovider -q -rN "
                                      f"--junitxml={report} {sel} >/dev/null 2>&1; true", timeout=timeout)
        if getattr(out, "timed_out", False):
            return None, "timeout"
        root = _parse_junit(_read_report(sandbox, report))
        if root is None:
            return None, "no_report"
        results.update(_junit_outcomes(root))
    return results, ""


def _run_go(sandbox: Any, timeout: float) -> tuple[dict[str, bool] | None, str]:
    out = command_output(sandbox, "go test -json ./... 2>/dev/null > /tmp/ts-go.json; true", timeout=timeout)
    if getattr(out, "timed_out", False):
        return None, "timeout"
    text = _read_report(sandbox, "/tmp/ts-go.json")
    if text is None:
        return None, "no_report"
    res: dict[str, bool] = {}
    for line in text.splitlines():
        try:
            ev = json.loads(line)
        except ValueError:
            continue
        name = ev.get("Test")
        if name and ev.get("Action") in ("pass", "fail", "skip"):
            res[name] = ev["Action"] == "pass"
    return res, ""


def grade(sandbox: Any, task: Task, *, restore_tests: bool = True, check_regressions: bool = True,
          timeout: float = 1800.0) -> Verdict:
    """Reward 1 iff every FAIL_TO_PASS test passes and (optionally) no PASS_TO_PASS test regresses."""
    f2p = parse_test_ids(task.fail_to_pass)
    p2p = parse_test_ids(task.pass_to_pass) if check_regressions else []
    if restore_tests and getattr(sandbox, "bug_base", None):
        files = sorted({t.split("::")[0] for t in f2p + p2p if "::" in t})
        if files:
            sandbox.exec(f"git checkout -q {sandbox.bug_base} -- " + " ".join(shlex.quote(f) for f in files) +
                         " 2>/dev/null; true")
    wanted = f2p + p2p
    if task.test_framework == "go":
        res, why = _run_go(sandbox, timeout)
    else:
        res, why = _run_pytest(sandbox, wanted, timeout) if wanted else ({}, "")
    if res is None:
        return Verdict(0.0, missing=list(wanted), n_pass_to_pass=len(p2p), reason=why)
    passed = [t for t in f2p if res.get(t) is True]
    failed = [t for t in f2p if res.get(t) is False]
    missing = [t for t in f2p if t not in res]
    regressed = [t for t in p2p if res.get(t) is False or t not in res]
    ok = bool(f2p) and len(passed) == len(f2p) and not regressed
    reason = "pass" if ok else ("missing" if missing else ("regressed" if regressed else "fail"))
    return Verdict(1.0 if ok else 0.0, passed, failed, missing, regressed, len(p2p), reason)


def run_tests(sandbox: Any, task: Task, *, restore_tests: bool = True, check_regressions: bool = True) -> float:
    """Binary reward (a group without reward spread is then exactly a zero-advantage group)."""
    return grade(sandbox, task, restore_tests=restore_tests, check_regressions=check_regressions).reward


def grade_isolated(policy_sandbox: Any, task: Task, verifier_factory: Callable[[str, str], Any], *,
                   name: str = "verify", max_patch_bytes: int = 8 << 20) -> Verdict:
    """Capture the policy's patch on the host, apply it in a fresh verifier sandbox and grade there."""
    try:
        patch = capture_policy_patch(policy_sandbox, max_bytes=max_patch_bytes)
    except PolicyPatchRejected as exc:
        return Verdict(0.0, reason=f"patch_rejected: {exc}")
    box = new_sandbox(verifier_factory, task, name)
    try:
        box.start()
        if task.bug_patch:
            box.apply_bug_patch(task.bug_patch)
        if patch.strip():
            (Path(box.host_tmp) / "policy.patch").write_bytes(patch)
            out = box.exec_output("git apply --binary --whitespace=nowarn /tmp/policy.patch")
            if out.returncode != 0:
                return Verdict(0.0, reason="patch_does_not_apply")
        return grade(box, task)
    finally:
        box.close()


# ---------------------------------------------------------------------------- generation broker
@dataclass
class _GenRequest:
    prompt: list[int]
    seed: int | None
    max_tokens: int
    temperature: float
    done: threading.Event
    result: GenResult | None = None
    error: BaseException | None = None


class _GenerationBroker:
    """Coalesces outstanding per-rollout requests into one ``generate`` call on a dispatcher thread."""

    def __init__(self, engine: "BatchedRolloutEngine", *, linger_s: float = 0.002,
                 timings: BatchTimings | None = None) -> None:
        self.engine = engine
        self.linger_s = linger_s
        self.timings = timings
        self._q: queue.Queue = queue.Queue()
        self._thread: threading.Thread | None = None
        self._closed = False

    def start(self) -> "_GenerationBroker":
        self._thread = threading.Thread(target=self._loop, name="ts-generation-broker", daemon=True)
        self._thread.start()
        return self

    def close(self) -> None:
        self._closed = True
        self._q.put(None)
        if self._thread is not None:
            self._thread.join()

    def __enter__(self) -> "_GenerationBroker":
        return self.start()

    def __exit__(self, *exc) -> None:
        self.close()

    def submit(self, prompt: list[int], *, seed: int | None, max_tokens: int, temperature: float) -> GenResult:
        if self._closed:
            raise RuntimeError("generation broker is closed")
        req = _GenRequest(list(prompt), seed, max_tokens, temperature, threading.Event())
        self._q.put(req)
        req.done.wait()
        if req.error is not None:
            raise req.error
        return req.result

    def _collect(self) -> tuple[list[_GenRequest], bool]:
        first = self._q.get()
        if first is None:
            return [], True
        reqs = [first]
        deadline = time.perf_counter() + self.linger_s
        stop = False
        while True:
            try:
                nxt = self._q.get(timeout=max(0.0, deadline - time.perf_counter()))
            except queue.Empty:
                break
            if nxt is None:
                stop = True
                break
            reqs.append(nxt)
        return reqs, stop

    def _loop(self) -> None:
        while True:
            reqs, stop = self._collect()
            if reqs:
                self._serve(reqs)
            if stop:
                while not self._q.empty():
                    r = self._q.get_nowait()
                    if r is not None:
                        r.error = RuntimeError("generation broker closed")
                        r.done.set()
                return

    def _serve(self, reqs: list[_GenRequest]) -> None:
        by_temp: dict[float, list[_GenRequest]] = {}
        for r in reqs:
            by_temp.setdefault(r.temperature, []).append(r)
        for temp, group in by_temp.items():
            t0 = time.perf_counter()
            try:
                outs = self.engine.generate([r.prompt for r in group], max_tokens=[r.max_tokens for r in group],
                                            temperature=temp, seeds=[r.seed for r in group])
            except BaseException as exc:  # noqa: BLE001 - handed to every waiting worker
                for r in group:
                    r.error = exc
                    r.done.set()
                continue
            now = time.perf_counter()
            if self.timings is not None:
                self.timings.shared_generation_s += now - t0
                self.timings.shared_generation_batch_sizes.append(len(group))
                self.timings.shared_generation_prompt_tokens += sum(len(r.prompt) for r in group)
                self.timings.shared_generation_completion_tokens += sum(len(o.token_ids) for o in outs)
            for r, o in zip(group, outs):
                o.ready_at = now
                r.result = o
                r.done.set()


# ---------------------------------------------------------------------------- engine
class BatchedRolloutEngine:
    """vLLM offline engine + agent loop + grading; ``llm``/``tokenizer`` may be injected (tests, custom engines)."""

    def __init__(self, model_path: str | Path | None = None, *, tensor_parallel_size: int = 1,
                 max_model_len: int = 131072, gpu_memory_utilization: float = 0.65, enable_prefix_caching: bool = True,
                 seed: int = 0, enable_lora: bool = False, max_lora_rank: int = 32,
                 enable_chunked_prefill: bool | None = True, max_num_seqs: int | None = 16,
                 max_num_batched_tokens: int | None = None, llm: Any = None, tokenizer: Any = None) -> None:
        if isinstance(tensor_parallel_size, bool) or not isinstance(tensor_parallel_size, int) or \
                tensor_parallel_size < 1:
            raise ValueError(f"tensor_parallel_size must be a positive integer, not {tensor_parallel_size!r}")
        if llm is None:
            from vllm import LLM

            kw: dict[str, Any] = {}
            if enable_lora:
                kw.update(enable_lora=True, max_lora_rank=max_lora_rank, max_loras=1)
            if max_num_seqs is not None:
                kw["max_num_seqs"] = max_num_seqs
            if max_num_batched_tokens is not None:
                kw["max_num_batched_tokens"] = max_num_batched_tokens
            if enable_chunked_prefill is not None:
                kw["enable_chunked_prefill"] = enable_chunked_prefill
            llm = LLM(model=str(model_path), tensor_parallel_size=tensor_parallel_size, max_model_len=max_model_len,
                      gpu_memory_utilization=gpu_memory_utilization, enable_prefix_caching=enable_prefix_caching,
                      seed=seed, disable_log_stats=True, **kw)
        self.llm = llm
        self.tokenizer = tokenizer if tokenizer is not None else llm.get_tokenizer()
        self.max_model_len = max_model_len
        self.lora_request = None

    def encode(self, text: str) -> list[int]:
        return list(self.tokenizer.encode(text, add_special_tokens=False))

    def decode(self, ids: Sequence[int]) -> str:
        return self.tokenizer.decode(list(ids), skip_special_tokens=False)

    def generate(self, prompts: Sequence[Sequence[int]], *, max_tokens: int | Sequence[int] = 1024,
                 temperature: float = 1.0, top_p: float = 1.0, seeds: Sequence[int | None] | None = None
                 ) -> list[GenResult]:
        """One completion per token-id prompt, with the sampled token's logprob."""
        caps = [int(c) for c in max_tokens] if isinstance(max_tokens, Sequence) else [int(max_tokens)] * len(prompts)
        if len(caps) != len(prompts):
            raise ValueError(f"{len(caps)} max_tokens for {len(prompts)} prompts")
        custom = getattr(self.llm, "generate_token_ids", None)
        if custom is not None:  # an engine that speaks token ids natively (and test doubles)
            return [GenResult(list(ids), list(lps), text) for ids, lps, text in
                    custom([list(p) for p in prompts], caps, temperature, top_p, None if seeds is None else list(seeds))]
        from vllm import SamplingParams
        from vllm.inputs import TokensPrompt

        params = [SamplingParams(max_tokens=caps[i], temperature=temperature, top_p=top_p, top_k=-1,
                                 logprobs=0, seed=None if seeds is None or seeds[i] is None else int(seeds[i]))
                  for i in range(len(prompts))]
        outs = self.llm.generate([TokensPrompt(prompt_token_ids=list(p)) for p in prompts], params, use_tqdm=False,
                                 lora_request=self.lora_request)
        res = []
        for o in outs:
            c = o.outputs[0]
            ids = list(c.token_ids)
            lps = []
            for tok, d in zip(ids, c.logprobs or [{}] * len(ids)):
                v = d.get(tok) if d else None
                lps.append(float(getattr(v, "logprob", 0.0)) if v is not None else 0.0)
            res.append(GenResult(ids, lps, c.text, getattr(c, "finish_reason", "") or ""))
        return res

    # ------------------------------------------------------------------ prompts
    def _task_prompt(self, task: Task, box: Any, repo_context: bool, context_kwargs: dict | None) -> list[int]:
        if repo_context:
            tree, files = build_repo_context(box, task.problem_statement, **(context_kwargs or {}))
            user = CONTEXT_TEMPLATE.format(tree=tree, files=files, problem_statement=task.problem_statement)
        else:
            user = TASK_TEMPLATE.format(problem_statement=task.problem_statement)
        return self.encode(f"<|im_start|>system\n{SYSTEM_PROMPT}<|im_end|>\n<|im_start|>user\n{user}<|im_end|>\n")

    def _observation_ids(self, body: str) -> list[int]:
        return self.encode(f"<|im_end|>\n<|im_start|>user\n{body}<|im_end|>\n")

    # ------------------------------------------------------------------ groups
    def rollout_group(self, task: Task, *, schedule: str = "lockstep", **kwargs
                      ) -> tuple[list[Trajectory], BatchTimings]:
        if schedule not in ("lockstep", "async"):
            raise ValueError(f"unknown schedule {schedule!r}; expected one of ['async', 'lockstep']")
        return self._run_group(task, schedule=schedule, **kwargs)

    def rollout_groups(self, specs: Sequence[dict], *, schedule: str = "async",
                       max_concurrent_groups: int | None = None, gen_linger_s: float = 0.002, **common
                       ) -> list[tuple[list[Trajectory], BatchTimings]]:
        """Several groups; async groups share one broker so their rollouts batch together."""
        if schedule not in ("async", "lockstep"):
            raise ValueError(f"unknown schedule {schedule!r}")
        if not specs:
            return []
        if schedule == "lockstep":
            return [self.rollout_group(schedule="lockstep", **{**common, **s}) for s in specs]
        shared = BatchTimings(schedule="async")
        with _GenerationBroker(self, linger_s=gen_linger_s, timings=shared) as brk:
            workers = max_concurrent_groups or len(specs)
            with ThreadPoolExecutor(max_workers=workers) as pool:
                futs = [pool.submit(self._run_group, schedule="async", broker=brk, **{**common, **s}) for s in specs]
                out = [f.result() for f in futs]
        for _, t in out:
            t.shared_generation_s = shared.shared_generation_s
            t.shared_generation_batch_sizes = list(shared.shared_generation_batch_sizes)
            t.shared_generation_prompt_tokens = shared.shared_generation_prompt_tokens
            t.shared_generation_completion_tokens = shared.shared_generation_completion_tokens
        return out

    def _run_group(self, task: Task, *, schedule: str, group_size: int, group_id: int = 0, max_steps: int = 300,
                   max_tokens_per_step: int = 1024, max_generated_tokens: int = 16384,
                   max_observation_tokens: int = 4096, max_prompt_tokens: int = 16384, temperature: float = 1.0,
                   sandbox_prefix: str = "thundersync", base_seed: int = 0, tool_workers: int = 8,
                   repo_context: bool = True, score: bool = True, turn_open: str = "<|im_start|>assistant\n",
                   context_kwargs: dict | None = None, on_prompt=None, on_block=None, on_step=None,
                   on_trajectory_complete=None, on_verdict=None, sandbox_factory=None, grade_fn=None,
                   broker: _GenerationBroker | None = None, **_ignored) -> tuple[list[Trajectory], BatchTimings]:
        if isinstance(max_prompt_tokens, bool) or not isinstance(max_prompt_tokens, int) or max_prompt_tokens < 1:
            raise ValueError(f"max_prompt_tokens must be a positive integer, not {max_prompt_tokens!r}")
        if sandbox_factory is None:
            from thundersync_b200.rollout.docker_sandbox import DockerSandbox

            sandbox_factory = DockerSandbox
        score_fn = grade_fn or grade
        timings = BatchTimings(schedule=schedule)
        timings.verdict_at = [0.0] * group_size
        timings.trajectory_completed_at = [0.0] * group_size
        boxes = [new_sandbox(sandbox_factory, task, f"{sandbox_prefix}-{group_id}-{i}") for i in range(group_size)]
        lock = threading.Lock()
        try:
            with ThreadPoolExecutor(max_workers=max(1, min(tool_workers, group_size))) as pool:
                list(pool.map(lambda b: self._setup(b, task), boxes))
            prompt_ids = self._task_prompt(task, boxes[0], repo_context, context_kwargs)
            if len(prompt_ids) > max_prompt_tokens:
                raise ValueError(f"{task.instance_id}: the initial prompt is {len(prompt_ids)} tokens, over "
                                 f"max_prompt_tokens={max_prompt_tokens}")
            if on_prompt is not None:
                on_prompt(list(prompt_ids))
            open_ids = self.encode(turn_open)
            trajs = [Trajectory(task.instance_id, group_id, i, list(prompt_ids)) for i in range(group_size)]
            cfg = dict(max_steps=max_steps, max_tokens_per_step=max_tokens_per_step,
                       max_generated_tokens=max_generated_tokens, max_observation_tokens=max_observation_tokens,
                       temperature=temperature, base_seed=base_seed, group_id=group_id, open_ids=open_ids)
            t0 = time.perf_counter()

            def verdict(i: int) -> None:
                tv = time.perf_counter()
                v = score_fn(boxes[i], task) if score else 0.0
                reward, reason = (v.reward, v.reason) if isinstance(v, Verdict) else (float(v), "")
                with lock:
                    trajs[i].reward = reward
                    trajs[i].verdict_reason = reason
                    timings.verify_s += time.perf_counter() - tv
                    timings.verdict_at[i] = time.perf_counter()
                    if on_verdict is not None:
                        on_verdict(i, trajs[i])

            def emit_block(i, block):
                if on_block is not None:
                    with lock:
                        on_block([(i, block)])

            if schedule == "lockstep":
                self._lockstep(trajs, boxes, prompt_ids, cfg, timings, emit_block, on_step, on_trajectory_complete,
                               tool_workers)
                if score:
                    with ThreadPoolExecutor(max_workers=max(1, min(tool_workers, group_size))) as pool:
                        list(pool.map(verdict, range(group_size)))
            else:
                own = broker is None
                brk = broker or _GenerationBroker(self, timings=timings).start()
                try:
                    def work(i):
                        self._async_one(i, trajs[i], boxes[i], prompt_ids, cfg, timings, brk, lock, emit_block,
                                        on_step, on_trajectory_complete)
                        if score:
                            verdict(i)

                    with ThreadPoolExecutor(max_workers=group_size) as pool:
                        list(pool.map(work, range(group_size)))
                finally:
                    if own:
                        brk.close()
            timings.rollout_wall_s = time.perf_counter() - t0
            timings.graded_at = max(timings.verdict_at) if score else 0.0
            return trajs, timings
        finally:
            for b in boxes:
                try:
                    b.close()
                except Exception:  # noqa: BLE001 - close every sandbox
                    log.exception("closing sandbox failed")

    @staticmethod
    def _setup(box: Any, task: Task) -> None:
        box.start()
        if task.bug_patch:
            box.apply_bug_patch(task.bug_patch)
        if hasattr(box, "host_workdir"):
            try:
                capture_trusted_bug_tree(box)
            except Exception:  # noqa: BLE001 - a host without git still rolls out; grading then runs in place
                log.warning("trusted tree capture failed for %s", getattr(box, "name", box))

    def _turn(self, i, traj, box, g: GenResult, step_idx: int, prompt_len: int, cfg, emit_block, gen_s: float):
        """Record one generated action, run its tool, return (step, finished)."""
        open_ids = cfg["open_ids"]
        action = parse_action(g.text)
        term = "submit" if action == "submit" else ("max_steps" if step_idx == cfg["max_steps"] - 1 else None)
        emit_block(i, CommittedBlock(step_idx, "action", tuple(open_ids + g.token_ids),
                                     (False,) * len(open_ids) + (True,) * len(g.token_ids),
                                     g.ready_at or time.perf_counter(), term))
        observation, tool_s = None, 0.0
        if action is None:
            observation = PARSE_ERROR_OBSERVATION
        elif action != "submit":
            t1 = time.perf_counter()
            observation = truncate_observation_tokens(command_output(box, action), self.encode, self.decode,
                                                      cfg["max_observation_tokens"])
            tool_s = time.perf_counter() - t1
        step = Step(action or g.text[:200], observation or "", open_ids + g.token_ids,
                    [0.0] * len(open_ids) + list(g.logprobs), generation_s=gen_s, tool_s=tool_s,
                    prompt_len=prompt_len)
        if action == "submit":
            return step, True
        step.observation_token_ids = self._observation_ids(observation)
        emit_block(i, CommittedBlock(step_idx, "observation", tuple(step.observation_token_ids),
                                     (False,) * len(step.observation_token_ids), time.perf_counter()))
        return step, False

    def _async_one(self, i, traj, box, prompt_ids, cfg, timings, brk, lock, emit_block, on_step, on_complete):
        ctx = list(prompt_ids)
        generated, gen_total, tool_total, turns, tools = 0, 0.0, 0.0, 0, 0
        open_ids = cfg["open_ids"]
        for step_idx in range(cfg["max_steps"]):
            if len(ctx) >= self.max_model_len - cfg["max_tokens_per_step"] - len(open_ids):
                traj.finish_reason = "context_limit"
                break
            if generated >= cfg["max_generated_tokens"]:
                traj.finish_reason = "generation_limit"
                break
            prompt = ctx + open_ids
            t0 = time.perf_counter()
            g = brk.submit(prompt, seed=request_seed(cfg["base_seed"], cfg["group_id"], i, step_idx),
                           max_tokens=min(cfg["max_tokens_per_step"], cfg["max_generated_tokens"] - generated),
                           temperature=cfg["temperature"])
            gen_s = time.perf_counter() - t0
            gen_total += gen_s
            generated += len(g.token_ids)
            turns += 1
            step, done = self._turn(i, traj, box, g, step_idx, len(prompt), cfg, emit_block, gen_s)
            tool_total += step.tool_s
            tools += int(step.tool_s > 0)
            traj.steps.append(step)
            if on_step is not None:
                with lock:
                    on_step(step_idx, [(i, step)])
            if done:
                traj.finish_reason = "submit"
                break
            ctx += step.action_token_ids + step.observation_token_ids
        if not traj.finish_reason:
            traj.finish_reason = "max_steps"
        traj.completed_at = time.perf_counter()
        with lock:
            timings.trajectory_completed_at[i] = traj.completed_at
            timings.generation_s += gen_total
            timings.tool_s += tool_total
            timings.tool_calls += tools
            timings.model_rows += turns
            timings.logical_rows += turns
            timings.n_steps = max(timings.n_steps, turns)
            if on_complete is not None:
                on_complete(i, traj)

    def _lockstep(self, trajs, boxes, prompt_ids, cfg, timings, emit_block, on_step, on_complete, tool_workers):
        n = len(trajs)
        ctx = [list(prompt_ids) for _ in range(n)]
        generated = [0] * n
        live = list(range(n))
        open_ids = cfg["open_ids"]
        with ThreadPoolExecutor(max_workers=max(1, min(tool_workers, n))) as pool:
            for step_idx in range(cfg["max_steps"]):
                ready = []
                for i in live:
                    if len(ctx[i]) >= self.max_model_len - cfg["max_tokens_per_step"] - len(open_ids):
                        trajs[i].finish_reason = "context_limit"
                    elif generated[i] >= cfg["max_generated_tokens"]:
                        trajs[i].finish_reason = "generation_limit"
                    else:
                        ready.append(i)
                for i in live:
                    if i not in ready:
                        self._complete(i, trajs, timings, on_complete)
                live = ready
                if not live:
                    break
                t0 = time.perf_counter()
                outs = self.generate([ctx[i] + open_ids for i in live],
                                     max_tokens=[min(cfg["max_tokens_per_step"], cfg["max_generated_tokens"] -
                                                     generated[i]) for i in live],
                                     temperature=cfg["temperature"],
                                     seeds=[request_seed(cfg["base_seed"], cfg["group_id"], i, step_idx)
                                            for i in live])
                gen_s = time.perf_counter() - t0
                now = time.perf_counter()
                for o in outs:
                    o.ready_at = now
                timings.generation_s += gen_s
                timings.generation_batch_sizes.append(len(live))
                timings.model_rows += len(live)
                timings.logical_rows += len(live)
                timings.n_steps = step_idx + 1
                t1 = time.perf_counter()
                results = list(pool.map(lambda ig: self._turn(ig[0], trajs[ig[0]], boxes[ig[0]], ig[1], step_idx,
                                                              len(ctx[ig[0]]) + len(open_ids), cfg, emit_block,
                                                              gen_s), zip(live, outs)))
                timings.tool_s += time.perf_counter() - t1
                events, nxt = [], []
                for i, g, (step, done) in zip(live, outs, results):
                    generated[i] += len(g.token_ids)
                    timings.tool_calls += int(step.tool_s > 0)
                    trajs[i].steps.append(step)
                    events.append((i, step))
                    if done:
                        trajs[i].finish_reason = "submit"
                        self._complete(i, trajs, timings, on_complete)
                    else:
                        ctx[i] += step.action_token_ids + step.observation_token_ids
                        nxt.append(i)
                if on_step is not None:
                    on_step(step_idx, events)
                live = nxt
        for i in live:
            trajs[i].finish_reason = trajs[i].finish_reason or "max_steps"
            self._complete(i, trajs, timings, on_complete)

    @staticmethod
    def _complete(i, trajs, timings, on_complete):
        trajs[i].completed_at = time.perf_counter()
        timings.trajectory_completed_at[i] = trajs[i].completed_at
        if on_complete is not None:
            on_complete(i, trajs[i])
