"""Allocator-level gate: streamed turns must not retain each event's full prefix.

A concatenate-then-attend op saves every event's [ancestors | own] key/value
chain, so retention grows as the sum of prefixes. The streamed path keeps only
chunk references (the [ancestors | own] buffer attention reads is rebuilt in
the backward), so the marginal allocated bytes per turn must stay flat in the
turn index and the peak must be materially lower. Same gate as reference
tests/test_stream_memory_regression.py:147-151 (peak < 75% of the
concatenating path, second-half / first-half slope < 1.1 while the
concatenating path's is > 1.1), measured on ``torch.cuda.memory_allocated``.
"""

from __future__ import annotations

import gc

import pytest
import torch

from thundersync_b200.engine.streaming import StreamingRun
from thundersync_b200.models.qwen3 import PRESETS, Qwen3ForCausalLM

pytestmark = pytest.mark.gpu

VOCAB = 512
PROMPT_LEN = 96
TURN_LEN = 96
TURNS = 16


def _model():
    cfg = PRESETS["qwen3-1.7b"].with_(num_hidden_layers=2, hidden_size=256, intermediate_size=512,
                                      num_attention_heads=2, num_key_value_heads=2, head_dim=128,
                                      vocab_size=VOCAB)
    torch.manual_seed(0)
    with torch.device("cuda"):
        model = Qwen3ForCausalLM(cfg).to(torch.bfloat16)
    return model.eval()


def _lsq_slope(ys):
    n = len(ys)
    mx, my = (n - 1) / 2, sum(ys) / n
    sxx = sum((x - mx) ** 2 for x in range(n))
    return sum((x - mx) * (y - my) for x, y in zip(range(n), ys)) / sxx


def _half_slope_ratio(series):
    n = len(series)
    return _lsq_slope(series[n // 2:]) / _lsq_slope(series[: n // 2])


def _stream(model, *, chunked: bool, turns: int = TURNS):
    gen = torch.Generator().manual_seed(7)

    def tokens(n):
        return torch.randint(0, VOCAB, (n,), generator=gen).tolist()

    run = StreamingRun(model, chunked_sdpa=chunked)
    gc.collect()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    torch.cuda.reset_peak_memory_stats()
    base = torch.cuda.memory_allocated()
    run.open_group(0, tokens(PROMPT_LEN))
    series = []
    for _ in range(turns):
        scored = [True] * (TURN_LEN // 2) + [False] * (TURN_LEN - TURN_LEN // 2)
        run.append_turn(0, 0, tokens(TURN_LEN), scored)
        torch.cuda.synchronize()
        series.append(torch.cuda.memory_allocated() - base)
    peak = torch.cuda.max_memory_allocated() - base
    run.logprobs(0).float().sum().backward()  # the retained graph is usable at this shape on both paths
    run.close()
    del run
    model.zero_grad(set_to_none=True)
    gc.collect()
    torch.cuda.empty_cache()
    return peak, series


def test_streamed_retention_is_linear_not_sum_of_prefixes():
    model = _model()
    for warm in (False, True):
        _stream(model, chunked=warm, turns=2)
    peak_old, series_old = _stream(model, chunked=False)
    peak_new, series_new = _stream(model, chunked=True)
    ratio_old = _half_slope_ratio(series_old)
    ratio_new = _half_slope_ratio(series_new)
    print(f"\npeak over base: concatenating {peak_old / 2**20:.1f} MiB, streamed {peak_new / 2**20:.1f} MiB; "
          f"slope ratio concatenating {ratio_old:.3f}, streamed {ratio_new:.3f}")
    assert ratio_old > 1.1, f"the concatenating baseline did not grow (ratio {ratio_old:.3f}): shape too small"
    assert ratio_new < 1.1, f"streamed marginal bytes grow with turn index (ratio {ratio_new:.3f})"
    assert peak_new < 0.75 * peak_old, f"streamed peak {peak_new} not >25% below concatenating {peak_old}"
