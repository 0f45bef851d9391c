"""The agent's text contracts: the action a reply carries and how long observations are shortened.

Behaviour stated after reference tests/rollout/test_parse_action.py and
tests/rollout/test_observation_truncation.py, checked with cases of this package's own: the first fenced
``bash`` block is the action (closing fence alone on its line, trailing blanks allowed, backticks
inside a line do not close it, a block cut before its fence is no action); token truncation keeps
``max_tokens // 2`` tokens at each end, counts the elided tokens exactly, leaves short outputs alone
and refuses limits below two tokens.
"""

from __future__ import annotations

import pytest

from thundersync_b200.rollout.agent import parse_action, truncate_observation_tokens


@pytest.mark.parametrize("reply,action", [
    ("Checking.\n```bash\ngrep -rn foo lib/\n```\nnext I patch it", "grep -rn foo lib/"),
    ("```bash\t\npytest -x\n```\t \n", "pytest -x"),
    ("```bash\nfirst\n```\ntext\n```bash\nsecond\n```", "first"),
    ("no code here", None),
    ("```sh\nls\n```", None),
    ("```bash\npartial command\n``", None),
])
def test_the_first_bash_block_is_the_action(reply, action):
    assert parse_action(reply) == action


def test_backticks_inside_a_line_stay_in_the_command():
    body = "printf '%s\\n' 'use ```code``` here'\necho ``` inline"
    assert parse_action(f"```bash\n{body}\n```") == body


def _tok():
    # one token per character: exact counts are easy to state
    return (lambda s: [ord(c) for c in s]), (lambda ids: "".join(chr(i) for i in ids))


def test_short_observations_are_unchanged():
    enc, dec = _tok()
    assert truncate_observation_tokens("abcdef", enc, dec, max_tokens=6) == "abcdef"


def test_long_observations_keep_both_ends_and_count_the_elided_tokens():
    enc, dec = _tok()
    text = "".join(chr(ord("a") + i % 26) for i in range(100))
    out = truncate_observation_tokens(text, enc, dec, max_tokens=10)
    head, tail = out.split("\n\n... <")[0], out.split("> ...\n\n")[1]
    assert head == text[:5] and tail == text[-5:]
    assert "<90 tokens elided>" in out
    odd = truncate_observation_tokens(text, enc, dec, max_tokens=7)
    assert odd.startswith(text[:3]) and odd.endswith(text[-4:]) and "<93 tokens elided>" in odd


def test_limits_below_two_tokens_are_refused():
    enc, dec = _tok()
    with pytest.raises(ValueError):
        truncate_observation_tokens("abc", enc, dec, max_tokens=1)
