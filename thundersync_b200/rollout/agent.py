"""A bash-only SWE agent whose trajectories are token-exact and append-only (C46).

The model replies with one fenced ```bash block per turn and receives the
command's output. Trajectories are recorded as token ids, never re-rendered
through a chat template, so two rollouts share exactly the physical prefix
they share — which is what the trainer's segment forest compresses.

The task context is laid out most-shared first: the repository file tree
(identical for every task of a repository), then the retrieved source files
(overlapping across tasks of a repository), then the issue (unique)
(reference: src/thundersync/rollout/agent.py:1-505). The prompt wording here
is this package's own.
"""

from __future__ import annotations

import re
import shlex
from dataclasses import dataclass, field
from typing import Callable, Protocol, Sequence

from thundersync_b200.rollout.bounded_output import CommandOutput, command_output

__all__ = [
    "ACTION_RE", "CONTEXT_TEMPLATE", "ExecSandbox", "ORDERINGS", "RetrievedFile", "SOURCE_EXTENSIONS",
    "SYSTEM_PROMPT", "Step", "TASK_TEMPLATE", "TEST_FRAMEWORKS", "Task", "Trajectory", "build_repo_context",
    "detect_source_extensions", "extract_keywords", "order_retrieved_files", "parse_action", "render_files_block",
    "retrieve_repo_files", "truncate_observation", "truncate_observation_tokens",
]


class ExecSandbox(Protocol):
    def exec(self, command: str) -> str: ...


SYSTEM_PROMPT = """You are working in a software repository to fix a reported defect.
Each reply must contain exactly one shell command in a fenced block:
```bash
<command>
```
It runs from the repository root; you will see what it prints.
Investigate, make a minimal change, and check it. When you are done, reply with:
```bash
submit
```
"""

TASK_TEMPLATE = """The repository is checked out at /testbed. Resolve this report:
<issue>
{problem_statement}
</issue>
Start by reading the code involved."""

# Repository-invariant block first, then per-task retrieved files, then the issue.
CONTEXT_TEMPLATE = """Repository index for /testbed.
<file_tree>
{tree}
</file_tree>
<relevant_files>
{files}
</relevant_files>
Resolve this report:
<issue>
{problem_statement}
</issue>
The excerpts above are a starting point; confirm the behaviour before changing code."""

_STOP = {
    "the", "and", "for", "with", "that", "this", "from", "when", "then", "have", "does", "not", "but", "are",
    "was", "were", "which", "should", "would", "will", "can", "issue", "problem", "error", "bug", "code", "file",
    "line", "expected", "actual", "description", "example", "following", "here", "there",
}
_IDENT = re.compile(r"\b[A-Za-z_][A-Za-z0-9_]{3,}\b")
SOURCE_EXTENSIONS = ("py", "go", "js", "ts", "jsx", "tsx", "java", "rb", "rs", "c", "h", "cc", "cpp", "hpp", "cs",
                     "php", "scala", "kt", "swift", "m", "sh")
ORDERINGS = ("grep", "path")
TEST_FRAMEWORKS = ("pytest", "go")
# An action is the body of a ```bash fence. Only a line that is nothing but
# ``` (plus spaces or tabs) ends it: backticks in the middle of a command line
# -- say a heredoc that writes Markdown -- stay part of the command.
ACTION_RE = re.compile(r"```bash[ \t]*\n(.*?)^```[ \t]*$", re.DOTALL | re.MULTILINE)


def extract_keywords(problem_statement: str, limit: int = 12) -> list[str]:
    """Identifiers of the issue, most frequent first (longer first on ties)."""
    counts: dict[str, int] = {}
    for m in _IDENT.finditer(problem_statement):
        w = m.group(0)
        if w.lower() not in _STOP:
            counts[w] = counts.get(w, 0) + 1
    return [w for w, _ in sorted(counts.items(), key=lambda kv: (-kv[1], -len(kv[0])))[:limit]]


def detect_source_extensions(sandbox: ExecSandbox, top: int = 3) -> list[str]:
    """The repository's most common source extensions (``["py"]`` when none are found)."""
    alt = "|".join(SOURCE_EXTENSIONS)
    out = sandbox.exec("find . -type f -not -path './.git/*' -not -path './build/*' "
                       rf"| grep -Eo '\.({alt})$' | sort | uniq -c | sort -rn | head -{top}")
    exts = []
    for line in out.splitlines():
        bits = line.split(".")
        if len(bits) >= 2 and bits[-1].strip():
            exts.append(bits[-1].strip())
    return exts or ["py"]


@dataclass(frozen=True)
class RetrievedFile:
    path: str
    body: str


def order_retrieved_files(files: Sequence[RetrievedFile], *, ordering: str = "grep") -> list[RetrievedFile]:
    if ordering == "grep":
        return list(files)
    if ordering == "path":
        return sorted(files, key=lambda f: f.path)
    raise ValueError(f"unknown ordering {ordering!r}; expected one of {ORDERINGS}")


def render_files_block(files: Sequence[RetrievedFile]) -> str:
    return "\n\n".join(f"--- {f.path} ---\n{f.body}" for f in files) or "(no files matched)"


def _display(path: str) -> str:
    while path.startswith("./"):
        path = path[2:]
    return path


def retrieve_repo_files(sandbox: ExecSandbox, problem_statement: str, *, max_tree_entries: int = 400,
                        max_files: int = 6, max_file_chars: int = 8000,
                        extensions: list[str] | None = None) -> tuple[str, list[RetrievedFile]]:
    """The file tree and the files with the most keyword hits, in hit-count order."""
    exts = extensions or detect_source_extensions(sandbox)
    names = " -o ".join(f"-name {shlex.quote('*.' + e)}" for e in exts)
    tree = sandbox.exec(f"find . \\( {names} \\) -not -path './.git/*' -not -path './build/*' "
                        f"| sed 's|^\\./||' | sort | head -{max_tree_entries}").strip()
    files: list[RetrievedFile] = []
    kws = extract_keywords(problem_statement)
    if kws:
        include = " ".join(shlex.quote(f"--include=*.{e}") for e in exts)
        pattern = "|".join(re.escape(k) for k in kws)
        ranked = sandbox.exec(f"grep -rEc {shlex.quote(pattern)} {include} . 2>/dev/null | grep -v ':0$' "
                              f"| sort -t: -k2 -rn | head -{max_files} | cut -d: -f1").strip()
        for path in [p for p in ranked.splitlines() if p.strip()][:max_files]:
            body = command_output(sandbox, f"cat {shlex.quote(path)} 2>/dev/null")
            text = body.text if body.complete else body.rendered()
            if text.strip():
                files.append(RetrievedFile(_display(path), truncate_observation(body, max_file_chars)))
    return tree or "(empty)", files


def build_repo_context(sandbox: ExecSandbox, problem_statement: str, *, max_tree_entries: int = 400,
                       max_files: int = 6, max_file_chars: int = 8000, extensions: list[str] | None = None,
                       ordering: str = "grep") -> tuple[str, str]:
    """(file tree, rendered files block), computed once per group so it lands in the shared prefix."""
    if ordering not in ORDERINGS:
        raise ValueError(f"unknown ordering {ordering!r}; expected one of {ORDERINGS}")
    tree, files = retrieve_repo_files(sandbox, problem_statement, max_tree_entries=max_tree_entries,
                                      max_files=max_files, max_file_chars=max_file_chars, extensions=extensions)
    return tree, render_files_block(order_retrieved_files(files, ordering=ordering))


@dataclass
class Task:
    instance_id: str
    problem_statement: str
    image_name: str
    fail_to_pass: list[str] = field(default_factory=list)
    pass_to_pass: list[str] = field(default_factory=list)
    repo: str = ""
    bug_patch: str = ""
    """The diff that introduces the bug (SWE-smith convention), applied at sandbox setup."""
    test_framework: str = "pytest"
    requires_network: bool = False

    def __post_init__(self) -> None:
        if self.test_framework not in TEST_FRAMEWORKS:
            raise ValueError(f"unknown test_framework {self.test_framework!r}; expected one of {TEST_FRAMEWORKS}")


@dataclass
class Step:
    action: str
    observation: str
    action_token_ids: list[int] = field(default_factory=list)
    action_logprobs: list[float] = field(default_factory=list)
    observation_token_ids: list[int] = field(default_factory=list)
    generation_s: float = 0.0
    tool_s: float = 0.0
    prompt_len: int = 0


@dataclass
class Trajectory:
    task_id: str
    group_id: int
    rollout_id: int
    prompt_token_ids: list[int] = field(default_factory=list)
    steps: list[Step] = field(default_factory=list)
    reward: float = 0.0
    finish_reason: str = ""
    completed_at: float | None = None
    final_diff: str = ""
    verdict_reason: str = ""

    @property
    def token_ids(self) -> list[int]:
        out = list(self.prompt_token_ids)
        for s in self.steps:
            out += s.action_token_ids
            out += s.observation_token_ids
        return out

    @property
    def action_mask(self) -> list[bool]:
        """True exactly on policy-generated (trainable) tokens."""
        out = [False] * len(self.prompt_token_ids)
        for s in self.steps:
            out += [True] * len(s.action_token_ids)
            out += [False] * len(s.observation_token_ids)
        return out

    @property
    def logprobs(self) -> list[float]:
        out = [0.0] * len(self.prompt_token_ids)
        for s in self.steps:
            out += s.action_logprobs
            out += [0.0] * len(s.observation_token_ids)
        return out

    @property
    def turns(self) -> list[tuple[list[int], list[bool]]]:
        """(tokens, scored mask) per step: the action tokens scored, the observation not."""
        return [(s.action_token_ids + s.observation_token_ids,
                 [True] * len(s.action_token_ids) + [False] * len(s.observation_token_ids)) for s in self.steps]

    @property
    def n_action_tokens(self) -> int:
        return sum(len(s.action_token_ids) for s in self.steps)

    @property
    def generation_s(self) -> float:
        return sum(s.generation_s for s in self.steps)

    @property
    def tool_s(self) -> float:
        return sum(s.tool_s for s in self.steps)


def truncate_observation(text: str | CommandOutput, max_chars: int = 4000) -> str:
    """Keep both ends (what ran, what broke); an incomplete capture renders as its full text would."""
    if isinstance(text, CommandOutput):
        if text.complete:
            return truncate_observation(text.text, max_chars)
        half = max_chars // 2
        if half < 1 or text.chars <= max_chars:
            raise ValueError(f"an incomplete output of {text.chars} chars cannot render at {max_chars}")
        return f"{text.head(half)}\n\n... <{text.chars - max_chars} chars elided> ...\n\n{text.tail(half)}"
    if len(text) <= max_chars:
        return text
    half = max_chars // 2
    return f"{text[:half]}\n\n... <{len(text) - max_chars} chars elided> ...\n\n{text[-half:]}"


_WHOLE_CHARS = 1 << 16
_MARGIN = 64
_CHARS_PER_TOKEN = 4
_GROWTH = 4
_SEAM = 3


def _end_tokens(text: str, count: int, encode, *, tail: bool) -> tuple[list[int], int]:
    """Tokens of a char window at one end holding ``count`` + margin tokens (or the whole text)."""
    width = _CHARS_PER_TOKEN * (count + _MARGIN)
    while True:
        if width >= len(text):
            return encode(text), len(text)
        ids = encode(text[-width:] if tail else text[:width])
        if len(ids) >= count + _MARGIN:
            return ids, width
        width *= _GROWTH


def _clean(ids: list[int], text: str, decode, *, tail: bool) -> str:
    """Decode, dropping up to three tokens at the cut when a byte-level token split a character."""
    ok = text.endswith if tail else text.startswith
    for k in range(_SEAM + 1):
        piece = decode(ids[k:] if tail else ids[: len(ids) - k])
        if ok(piece):
            return piece
    return decode(ids)


def truncate_observation_tokens(output: str | CommandOutput, encode: Callable[[str], list[int]],
                                decode: Callable[[Sequence[int]], str], max_tokens: int = 4096) -> str:
    """First and last ``max_tokens // 2`` tokens; the marker counts elided tokens when the whole text was
    tokenized, else elided characters."""
    if max_tokens < 2:
        raise ValueError(f"max_tokens must be at least 2, not {max_tokens}")
    nh = max_tokens // 2
    nt = max_tokens - nh
    if isinstance(output, CommandOutput) and not output.complete:
        htext, ttext, total = output.kept_head(), output.kept_tail(), output.chars
        hids, _ = _end_tokens(htext, nh, encode, tail=False)
        tids, _ = _end_tokens(ttext, nt, encode, tail=True)
    else:
        text = output.text if isinstance(output, CommandOutput) else output
        htext = ttext = text
        total = len(text)
        if len(text) <= _WHOLE_CHARS:
            hids, hw = encode(text), len(text)
        else:
            hids, hw = _end_tokens(text, nh, encode, tail=False)
        whole = hids if hw >= len(text) else None
        if whole is None:
            tids, tw = _end_tokens(text, nt, encode, tail=True)
            if hw + tw >= len(text):
                whole = encode(text)
        if whole is not None:
            if len(whole) <= max_tokens:
                return text
            head = _clean(whole[:nh], text, decode, tail=False)
            tail = _clean(whole[-nt:], text, decode, tail=True)
            return f"{head}\n\n... <{len(whole) - nh - nt} tokens elided> ...\n\n{tail}"
    head = _clean(hids[:nh], htext, decode, tail=False)
    tail = _clean(tids[-nt:], ttext, decode, tail=True)
    return f"{head}\n\n... <{total - len(head) - len(tail)} chars elided> ...\n\n{tail}"


def parse_action(text: str) -> str | None:
    """The body of the first ```bash block, stripped; None without one."""
    m = ACTION_RE.search(text)
    return m.group(1).strip() if m else None
