"""accel helpers: fused log-prob API, operator ranges, capability trials, merged LoRA.

Reference behaviour: tests/test_accel.py, tests/test_accel_entropy.py,
tests/test_fused_lora.py, tests/test_kernel_capability.py of the reference
(fused == naive in value and gradient; merged LoRA == unfused to fp32
rounding; trials run once per key and record their outcome).
"""

from __future__ import annotations

import pytest
import torch

from thundersync_b200.accel import capability, operator_profiling as op
from thundersync_b200.accel.fused_logprob import (fused_logprob, fused_logprob_entropy, gathered_logprobs,
                                                  naive_logprobs)
from thundersync_b200.accel.fused_lora import fuse_merged_lora_forward, unfuse_merged_lora_forward
from thundersync_b200.models.lora import LoRALinear


def test_fused_logprob_matches_naive_value_and_grad():
    torch.manual_seed(0)
    h = torch.randn(10, 16, requires_grad=True)
    w = torch.randn(50, 16, requires_grad=True)
    ids = torch.randint(0, 50, (10,))
    mask = torch.ones(10, dtype=torch.bool)
    got = gathered_logprobs(h, w, ids, mask, chunk=3)
    want = naive_logprobs(h, w, ids, mask)
    assert torch.allclose(got, want, atol=1e-5)
    g1 = torch.autograd.grad(got.sum(), (h, w))
    g2 = torch.autograd.grad(want.sum(), (h, w))
    for a, b in zip(g1, g2):
        assert torch.allclose(a, b, atol=1e-5)
    assert got[0] == 0


def test_fused_entropy_matches_softmax_entropy():
    torch.manual_seed(1)
    h = torch.randn(6, 8, requires_grad=True)
    w = torch.randn(30, 8)
    t = torch.randint(0, 30, (6,))
    lp, ent = fused_logprob_entropy(h, w, t, chunk=4)
    logp = torch.log_softmax(h @ w.t(), -1)
    assert torch.allclose(lp, logp.gather(-1, t[:, None]).squeeze(-1), atol=1e-5)
    ref_ent = -(logp.exp() * logp).sum(-1)
    assert torch.allclose(ent, ref_ent, atol=1e-5)
    (ga,) = torch.autograd.grad(ent.sum(), h)
    (gb,) = torch.autograd.grad(ref_ent.sum(), h)
    assert torch.allclose(ga, gb, atol=1e-4)
    with pytest.raises(ValueError):
        fused_logprob(h[None], w, t)


def test_operator_ranges(monkeypatch):
    monkeypatch.setattr(op, "_state", {"mode": None, "roles": {}})
    monkeypatch.setenv(op.PROFILE_RANGES_ENV, "off")
    assert op.operator_range("x") is op.operator_range("y")
    assert not op.operator_profiling_enabled()
    op.configure_operator_profiling("kineto", device_roles={"cpu": "learner"})
    assert op.device_role("cpu") == "learner"
    assert op.range_name("fwd", layer=3, skip=None, tag="a|b") == "thundersync::fwd|layer=3|tag=a/b"
    with torch.profiler.profile() as prof:
        with op.operator_range("block", n=2):
            torch.ones(3).sum()
    assert any(e.name == "thundersync::block|n=2" for e in prof.events())
    with pytest.raises(ValueError):
        op.configure_operator_profiling("loud")
    op.configure_operator_profiling("off")


def test_capability_trials_cpu():
    capability.reset_kernel_probes()
    calls = []
    assert not capability.kernel_runs("k", torch.zeros(1), 0, lambda d, t, s: calls.append(1))
    assert calls == [] and capability.kernel_probe_records() == []


def test_merged_lora_matches_unfused_and_restores():
    torch.manual_seed(0)
    model = torch.nn.Sequential(LoRALinear(torch.nn.Linear(12, 20, bias=False), 4, 8.0))
    with torch.no_grad():
        model[0].lora_B["default"].weight.normal_()
    base0 = model[0].base_layer.weight.detach().clone()
    x = torch.randn(5, 12)
    y0 = model(x)
    a, b = model[0].lora_A["default"].weight, model[0].lora_B["default"].weight
    ga0 = torch.autograd.grad(y0.square().sum(), (a, b))
    assert fuse_merged_lora_forward(model) == 1
    y1 = model(x)
    ga1 = torch.autograd.grad(y1.square().sum(), (a, b))
    assert torch.allclose(y0, y1, atol=1e-5)
    for p, q in zip(ga0, ga1):
        assert torch.allclose(p, q, atol=1e-4)
    assert unfuse_merged_lora_forward(model) == 1
    assert torch.allclose(model[0].base_layer.weight, base0, atol=1e-6)
