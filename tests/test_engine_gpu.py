"""Streaming GRPO on CUDA (native kernels, bf16) against the CPU fp32 oracle."""

from __future__ import annotations

import copy

import pytest
import torch

from tests.grpo_fixtures import EPS, advantages, make_batch
from tests.reference_model import reference_logprobs
from thundersync_b200.engine.streaming import StreamingRun
from thundersync_b200.grpo.reward_linear import RewardLinearBackward
from thundersync_b200.models.qwen3 import PRESETS, Qwen3ForCausalLM

pytestmark = pytest.mark.gpu

CFG = PRESETS["qwen3-1.7b"].with_(num_hidden_layers=2, hidden_size=256, intermediate_size=512,
                                  num_attention_heads=4, num_key_value_heads=2, vocab_size=2048)


def _grads_reference(model, batch):
    model.zero_grad(set_to_none=True)
    total = 0.0
    for g, prompt, trajs in batch:
        adv = advantages([r for _, _, r in trajs])
        for (tid, turns, _), a in zip(trajs, adv):
            total = total + a * reference_logprobs(model, prompt, turns).sum()
    total.backward()
    return {n: p.grad.detach().clone() for n, p in model.named_parameters()}


@pytest.mark.parametrize("binary,stream_turns", [(True, False), (False, True)])
def test_gpu_streamed_grpo_matches_fp32_oracle(binary, stream_turns):
    torch.manual_seed(0)
    model = Qwen3ForCausalLM(CFG)
    batch, order = make_batch(0, vocab=CFG.vocab_size, lo=40, hi=200, prompt_len=64, multi_turn=stream_turns)
    ref = _grads_reference(copy.deepcopy(model), batch)
    gm = copy.deepcopy(model).to("cuda", torch.bfloat16)
    run = StreamingRun(gm, boundary_cut=True, stream_turns=stream_turns)
    bw = RewardLinearBackward(run, gm, eps=EPS, source_offload_mode="device_resident", source_offload_device=None)
    if binary:
        bw.configure_binary_rewards()
    for g, prompt, trajs in batch:
        bw.open_group(g, prompt, [t for t, _, _ in trajs])
    for g, (tid, turns, reward) in order:
        for tk, sc in turns:
            run.append_turn(g, tid, tk, sc)
        bw.close_trajectory(tid, reward)
    for g, _, _ in batch:
        bw.close_group(g)
    bw.assert_safe_to_step()
    num = den = 0.0
    for n, p in gm.named_parameters():
        a, b = p.grad.float().cpu(), ref[n]
        num += float((a - b).pow(2).sum())
        den += float(b.pow(2).sum())
        cos = torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0)
        assert cos > 0.98, (n, float(cos))
    assert (num / den) ** 0.5 < 0.06


@pytest.mark.parametrize("prompt_len,cont_len", [(128, 200), (96, 75)])
def test_gpu_single_node_layer_matches_op_by_op(prompt_len, cont_len):
    """On CUDA the one-node dense layer (ancestor and own keys in one buffer, outputs written in place,
    padded pack rows) agrees with the op-by-op path, including gradients that reach the prompt's K/V."""
    from thundersync_b200.engine.layers import Executor, Segment

    cfg = PRESETS["qwen3-1.7b"].with_(num_hidden_layers=2, hidden_size=512, intermediate_size=1024,
                                      num_attention_heads=4, num_key_value_heads=2, head_dim=128, vocab_size=1024)
    torch.manual_seed(3)
    model = Qwen3ForCausalLM(cfg).to("cuda", torch.bfloat16)
    ids = torch.randint(0, cfg.vocab_size, (prompt_len + cont_len,), device="cuda")
    pos = torch.arange(prompt_len + cont_len, device="cuda")
    from thundersync_b200.engine import dense_layer as DL
    from thundersync_b200.engine.streaming import arena_for

    arena = arena_for(model)
    res = []
    for fused, native in ((True, True), (False, False), (True, False)):
        model.zero_grad(set_to_none=True)
        ex = Executor(model, arena)
        ex.fused_layers = fused
        DL.NATIVE = native
        def padded(x):  # pack rows padded to a multiple of 128 as the streaming engine pads them
            return torch.cat((x, x.new_zeros((-x.shape[0]) % 128)))

        h0, st0 = ex.run(padded(ids[:prompt_len]), padded(pos[:prompt_len]), [Segment(0, prompt_len, [])])
        past = st0[0]
        h1, _ = ex.run(padded(ids[prompt_len:]), padded(pos[prompt_len:]),
                       [Segment(0, cont_len, [([k], [v]) for (k, v) in past])])
        h0, h1 = h0[:prompt_len], h1[:cont_len]
        (h0.float().square().mean() + h1.float().pow(3).mean()).backward()
        res.append((h1.detach().float(), {n: p.grad.float().clone() for n, p in model.named_parameters()
                                          if p.grad is not None}))
    DL.NATIVE = True
    # the C++-driven layer issues the same kernels as the Python-driven one: bitwise equal
    assert torch.equal(res[0][0], res[2][0])
    for n in res[0][1]:
        assert torch.equal(res[0][1][n], res[2][1][n]), n
    assert float((res[0][0] - res[1][0]).norm() / res[1][0].norm()) < 2e-2
    assert res[0][1].keys() == res[1][1].keys()
    for n in res[0][1]:
        a, b = res[0][1][n], res[1][1][n]
        assert float((a - b).norm() / b.norm().clamp_min(1e-12)) < 3e-2, n


def _gpu_grads(model, batch, order, rung):
    model.zero_grad(set_to_none=True)
    run = StreamingRun(model, boundary_cut=True, stream_turns=False, rebuild_block_tokens=64)
    orig = run.rebuild_logprobs
    run.rebuild_logprobs = lambda ids, **k: orig(ids, **{**k, "executor": rung})
    bw = RewardLinearBackward(run, model, eps=EPS, source_offload_mode="device_resident", source_offload_device=None)
    for g, prompt, trajs in batch:
        bw.open_group(g, prompt, [t for t, _, _ in trajs])
    for g, (tid, turns, reward) in order:
        for tk, sc in turns:
            run.append_turn(g, tid, tk, sc)
        bw.close_trajectory(tid, reward)
    for g, _, _ in batch:
        bw.close_group(g)
    bw.assert_safe_to_step()
    return {n: p.grad.detach().float().clone() for n, p in model.named_parameters()}, run


def test_gpu_checkpoint_inputs_parked_on_host_match_plain():
    """The lowest rung of the rebuild ladder (checkpoint inputs in page-locked host memory) on CUDA."""
    torch.manual_seed(1)
    model = Qwen3ForCausalLM(CFG).to("cuda", torch.bfloat16)
    batch, order = make_batch(1, vocab=CFG.vocab_size, lo=40, hi=200, prompt_len=64)
    ref, _ = _gpu_grads(model, batch, order, "plain")
    got, run = _gpu_grads(model, batch, order, "checkpoint_host")
    diag = run.rebuild_checkpoint_offload_diagnostics()
    assert diag["host_rebuilds"] > 0 and diag["write_bytes"] > 0 and diag["read_bytes"] == diag["write_bytes"]
    for n in ref:
        scale = ref[n].abs().max().clamp_min(1e-6)
        assert float((got[n] - ref[n]).abs().max() / scale) < 2e-2, n
    rep = run.turn_memory_report
    assert rep["windows"]["rebuild/checkpoint_host"]["calls"] > 0


@pytest.mark.parametrize("options", [
    {"source_offload_device": "cpu", "source_offload_mode": "pinned_nonblocking",
     "source_offload_window_bytes": 1 << 20, "source_offload_pinned_windows": 3},
    {"source_offload_device": "cpu", "source_offload_mode": "pinned_nonblocking", "statistic_keep_source_dtype": True},
    {"source_offload_device": "cpu", "source_offload_mode": "blocking", "source_offload_hbm_threshold": 0.999},
])
def test_gpu_host_statistics_match_device_statistics(options, tmp_path):
    """Host-resident statistics (windowed device->host folds, host->device combine) give the device result."""
    torch.manual_seed(2)
    model = Qwen3ForCausalLM(CFG).to("cuda", torch.bfloat16)
    batch, order = make_batch(2, vocab=CFG.vocab_size, lo=40, hi=200, prompt_len=64)

    def grads(**kw):
        model.zero_grad(set_to_none=True)
        run = StreamingRun(model, boundary_cut=True, stream_turns=False)
        bw = RewardLinearBackward(run, model, eps=EPS, **kw)
        for g, prompt, trajs in batch:
            bw.open_group(g, prompt, [t for t, _, _ in trajs])
        for g, (tid, turns, reward) in order:
            for tk, sc in turns:
                run.append_turn(g, tid, tk, sc)
            bw.close_trajectory(tid, reward)
        for g, _, _ in batch:
            bw.close_group(g)
        bw.assert_safe_to_step()
        return {n: p.grad.detach().float().clone() for n, p in model.named_parameters()}, bw.source_offload_report

    ref, _ = grads(source_offload_mode="device_resident", source_offload_device=None)
    got, report = grads(source_spill_directory=str(tmp_path), **options)
    if options["source_offload_mode"] == "blocking":
        assert report["device_groups_below_hbm_threshold"] > 0
    else:
        assert report["host_fold"]["folds"] > 0 and report["host_fold"]["combines"] > 0
    tol = 2e-2  # both arrive as bf16 .grad (fp32 sums in different orders, one rounding each)
    for n in ref:
        scale = ref[n].abs().max().clamp_min(1e-6)
        assert float((got[n] - ref[n]).abs().max() / scale) < tol, n
