"""Test doubles for the rollout layer: a host-directory sandbox, a fake docker CLI, a fake LLM."""

from __future__ import annotations

import os
import shutil
import sys
import tempfile
from pathlib import Path

from thundersync_b200.rollout.bounded_output import CommandOutput, run_bounded

FAKE_DOCKER = r'''#!/usr/bin/env python3
import json, os, shutil, subprocess, sys
state = os.environ["FAKE_DOCKER_STATE"]
db = os.path.join(state, "containers.json")
cons = json.load(open(db)) if os.path.exists(db) else {}
def save(): json.dump(cons, open(db, "w"))
a = sys.argv[1:]
if a[0] == "version":
    print("27.0.0-fake"); sys.exit(0)
if a[:2] == ["image", "inspect"]:
    img = a[-1]; d = os.path.join(state, "images", img)
    if os.path.isdir(d): print("sha256:" + img.replace(":", "-")); sys.exit(0)
    sys.exit(1)
if a[0] == "create":
    cons[a[a.index("--name") + 1]] = {"image": a[-2], "mounts": {}}; save(); sys.exit(0)
if a[0] == "cp":
    name, path = a[1].split(":", 1)
    shutil.copytree(os.path.join(state, "images", cons[name]["image"]), a[2]); sys.exit(0)
if a[0] == "rm":
    for n in a[1:]:
        cons.pop(n, None)
    save(); sys.exit(0)
if a[0] == "run":
    name = a[a.index("--name") + 1]; mounts = {}
    labels = [a[i + 1] for i, x in enumerate(a) if x == "--label"]
    for i, x in enumerate(a):
        if x == "-v":
            h, c = a[i + 1].split(":"); mounts[c] = h
    cons[name] = {"image": a[-3], "mounts": mounts, "labels": labels, "args": a}; save(); print("cid"); sys.exit(0)
if a[0] == "ps":
    want = [a[i + 1].split("=", 1)[1].split("=", 1) for i, x in enumerate(a) if x == "--filter"]
    for n, c in cons.items():
        labs = dict(l.split("=", 1) for l in c.get("labels", []))
        if all(labs.get(k) == v for k, v in want):
            print(n)
    sys.exit(0)
if a[0] == "exec":
    rest = a[1:]; wd = None
    if rest[0] == "-w":
        wd = rest[1]; rest = rest[2:]
    name, cmd = rest[0], rest[1:]
    m = cons[name]["mounts"]
    joined = " ".join(cmd)
    if "kill -9 -1" in joined or cmd[0] == "chown":
        sys.exit(0)  # never signal or chown the host
    import re
    pat = re.compile("|".join(re.escape(c) for c in sorted(m, key=len, reverse=True)) + r"(?=/|\b|$)")
    def fix(s):
        return pat.sub(lambda mt: m[mt.group(0)], s) if m else s
    cmd = [fix(x) for x in cmd]
    sys.exit(subprocess.call(cmd, cwd=m.get(wd, None) if wd else None))
sys.exit(2)
'''


def install_fake_docker(tmp: Path, images: dict[str, dict[str, str]]) -> dict[str, str]:
    state = tmp / "docker-state"
    for img, files in images.items():
        root = state / "images" / img
        for rel, text in files.items():
            p = root / rel
            p.parent.mkdir(parents=True, exist_ok=True)
            p.write_text(text)
    exe = tmp / "fake-docker"
    exe.write_text(FAKE_DOCKER.replace("#!/usr/bin/env python3", "#!" + sys.executable))
    exe.chmod(0o755)
    return {"FAKE_DOCKER_STATE": str(state), "THUNDERSYNC_DOCKER_BIN": str(exe),
            "THUNDERSYNC_SANDBOX_SCRATCH": str(tmp / "scratch")}


class LocalSandbox:
    """A host directory initialised as a git repository; commands run with bash in it."""

    def __init__(self, image: str, name: str, files: dict[str, str] | None = None) -> None:
        self.image, self.name = image, name
        self.files = files if files is not None else {"mod.py": "def f():\n    return 1\n"}
        self.requires_network = False
        self.host_root: Path | None = None
        self.host_workdir: Path | None = None
        self.host_tmp: Path | None = None
        self.bug_base = None
        self.closed = False
        self.commands: list[str] = []

    def start(self) -> None:
        self.host_root = Path(tempfile.mkdtemp(prefix="ts-local-"))
        self.host_workdir = self.host_root / "work"
        self.host_tmp = self.host_root / "tmp"
        self.host_workdir.mkdir()
        self.host_tmp.mkdir()
        for rel, text in self.files.items():
            (self.host_workdir / rel).write_text(text)
        self.exec("git init -q && git add -A && git -c user.name=t -c user.email=t@x commit -qm init")

    def exec_output(self, command: str, *, timeout: float | None = None, keep_bytes: int | None = None,
                    memory_guard=None, write_guard=None) -> CommandOutput:
        self.commands.append(command)
        run = run_bounded(["bash", "-c", command], timeout=timeout or 60, cwd=self.host_workdir,
                          keep_bytes=keep_bytes or (1 << 20), kill_bytes=max(keep_bytes or 0, 8 << 20),
                          env={**os.environ, "TMPDIR": str(self.host_tmp)}, memory_guard=memory_guard,
                          write_guard=write_guard)
        return CommandOutput.from_run(run)

    def exec(self, command: str) -> str:
        return str(self.exec_output(command))

    def apply_bug_patch(self, patch: str) -> None:
        pass

    def scratch_mounts(self):
        return {self.host_workdir: "/testbed", self.host_tmp: "/tmp"}

    def close(self) -> None:
        self.closed = True
        if self.host_root is not None:
            shutil.rmtree(self.host_root, ignore_errors=True)


class FakeTokenizer:
    """Byte-level: one token per UTF-8 byte."""

    def encode(self, text: str, add_special_tokens: bool = False) -> list[int]:
        return list(text.encode())

    def decode(self, ids, skip_special_tokens: bool = False) -> str:
        return bytes(ids).decode(errors="replace")


class FakeLLM:
    """Deterministic in (prompt, seed): turn k of a rollout writes a file, then submits."""

    def __init__(self) -> None:
        self.calls: list[int] = []

    def get_tokenizer(self):
        return FakeTokenizer()

    def generate_token_ids(self, prompts, caps, temperature, top_p, seeds):
        self.calls.append(len(prompts))
        out = []
        for p, cap, seed in zip(prompts, caps, seeds):
            turns = bytes(p).count(b"<|im_start|>assistant")
            if turns >= 3:
                text = "done\n```bash\nsubmit\n```"
            else:
                text = f"step\n```bash\necho {seed % 997} >> out.txt && cat out.txt\n```"
            ids = list(text.encode())[:cap]
            out.append((ids, [-0.5] * len(ids), bytes(ids).decode(errors="replace")))
        return out
