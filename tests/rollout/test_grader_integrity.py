"""The grader never scores correct work as failure, nor broken work as success.

A false negative silently changes how many rollouts of a group succeeded,
which shifts the group's mean and spread and so the advantage of every
rollout in it. The grader therefore reads pytest's JUnit report, never its
console text. Reference behaviour: tests/rollout/test_grader_integrity.py of
the reference, which runs the same classes of case inside docker images; here
each case runs real pytest in a throwaway git repository on the host
(``LocalSandbox``), so no container runtime is needed.
"""

from __future__ import annotations

import pytest

from tests.rollout.fakes import LocalSandbox
from thundersync_b200.rollout.agent import Task
from thundersync_b200.rollout.engine import grade, run_tests


def _box(files: dict[str, str]) -> LocalSandbox:
    box = LocalSandbox("local", "grader", files={"conftest.py": "", **files})
    box.start()
    return box


def _task(f2p, p2p=()):
    return Task("synthetic", "", "local", fail_to_pass=list(f2p), pass_to_pass=list(p2p))


@pytest.fixture
def sandbox_factory():
    made = []

    def make(files):
        box = _box(files)
        made.append(box)
        return box

    yield make
    for box in made:
        box.close()


def test_passing_test_that_warns_about_an_error_scores_one(sandbox_factory):
    box = sandbox_factory({"test_w.py": "import warnings\n\ndef test_ok():\n"
                                        "    warnings.warn('ValueError is deprecated')\n    assert True\n"})
    v = grade(box, _task(["test_w.py::test_ok"]), restore_tests=False)
    assert v.reward == 1.0, (v.reason, v.failed, v.missing)


def test_passing_test_that_prints_failure_words_scores_one(sandbox_factory):
    box = sandbox_factory({"test_p.py": "def test_ok():\n    print('FAILED ERROR Traceback AssertionError')\n"})
    assert run_tests(box, _task(["test_p.py::test_ok"]), restore_tests=False) == 1.0


def test_failing_test_scores_zero_and_is_named(sandbox_factory):
    box = sandbox_factory({"test_f.py": "def test_bad():\n    assert 1 == 2\n\ndef test_good():\n    pass\n"})
    v = grade(box, _task(["test_f.py::test_bad", "test_f.py::test_good"]), restore_tests=False)
    assert v.reward == 0.0 and v.failed == ["test_f.py::test_bad"] and v.passed == ["test_f.py::test_good"]


def test_a_missing_test_is_not_a_pass(sandbox_factory):
    box = sandbox_factory({"test_m.py": "def test_here():\n    pass\n"})
    v = grade(box, _task(["test_m.py::test_here", "test_m.py::test_gone"]), restore_tests=False)
    assert v.reward == 0.0 and "test_m.py::test_gone" in v.missing


def test_collection_error_scores_zero(sandbox_factory):
    box = sandbox_factory({"test_c.py": "def test_ok(:\n    pass\n"})
    assert grade(box, _task(["test_c.py::test_ok"]), restore_tests=False).reward == 0.0


def test_skipped_and_xfailed_targets_are_not_passes(sandbox_factory):
    box = sandbox_factory({"test_s.py": "import pytest\n\n@pytest.mark.skip(reason='no')\ndef test_skip():\n"
                                        "    pass\n\n@pytest.mark.xfail\ndef test_xf():\n    assert False\n"})
    assert grade(box, _task(["test_s.py::test_skip"]), restore_tests=False).reward == 0.0
    assert grade(box, _task(["test_s.py::test_xf"]), restore_tests=False).reward == 0.0


def test_parametrized_and_class_ids(sandbox_factory):
    body = ("import pytest\n\n@pytest.mark.parametrize('x', [1, 'a b'])\ndef test_p(x):\n    assert x\n\n"
            "class TestK:\n    def test_m(self):\n        pass\n")
    box = sandbox_factory({"test_q.py": body})
    ids = ["test_q.py::test_p[1]", "test_q.py::test_p[a b]", "test_q.py::TestK::test_m"]
    v = grade(box, _task(ids), restore_tests=False)
    assert v.reward == 1.0, (v.reason, v.missing, v.failed)


def test_regressions_gate_the_reward(sandbox_factory):
    box = sandbox_factory({"test_r.py": "def test_fixed():\n    pass\n\ndef test_kept():\n    assert False\n"})
    task = _task(["test_r.py::test_fixed"], ["test_r.py::test_kept"])
    v = grade(box, task, restore_tests=False)
    assert v.reward == 0.0 and v.regressed == ["test_r.py::test_kept"]
    assert grade(box, task, restore_tests=False, check_regressions=False).reward == 1.0


def test_no_targets_is_never_a_pass(sandbox_factory):
    box = sandbox_factory({"test_e.py": "def test_ok():\n    pass\n"})
    assert grade(box, _task([]), restore_tests=False).reward == 0.0


def test_reports_with_a_doctype_or_entities_are_malformed():
    from thundersync_b200.rollout.engine import _parse_junit

    good = '<testsuites><testsuite><testcase classname="test_a" name="test_x"/></testsuite></testsuites>'
    assert _parse_junit(good) is not None
    evil = ('<?xml version="1.0"?><!DOCTYPE r [<!ENTITY a "aaaa">]>'
            '<testsuites><testsuite><testcase classname="test_a" name="&a;"/></testsuite></testsuites>')
    assert _parse_junit(evil) is None and _parse_junit("") is None and _parse_junit("<broken") is None


def test_report_paths_are_fresh_per_grade(sandbox_factory):
    box = sandbox_factory({"test_o.py": "def test_ok():\n    pass\n"})
    grade(box, _task(["test_o.py::test_ok"]), restore_tests=False)
    grade(box, _task(["test_o.py::test_ok"]), restore_tests=False)
    paths = {c.split("--junitxml=")[1].split()[0] for c in box.commands if "--junitxml=" in c}
    assert len(paths) == 2
