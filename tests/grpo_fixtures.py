"""Shared fixtures for GRPO tests: the config-1 tiny model and batch."""

from __future__ import annotations

import random

import torch

from thundersync_b200.models.qwen3 import PRESETS, Qwen3ForCausalLM

EPS = 1e-6


def build_model(seed: int = 0, dtype=torch.float32, device="cpu", cfg=None):
    torch.manual_seed(seed)
    cfg = cfg or PRESETS["tiny"]
    with torch.device(device):
        m = Qwen3ForCausalLM(cfg)
    return m.to(dtype=dtype)


def make_batch(seed: int = 0, groups: int = 2, per_group: int = 4, prompt_len: int = 16,
               lo: int = 8, hi: int = 32, vocab: int = 512, multi_turn: bool = False):
    """Config 1: prompt ids uniform, completion length uniform in [lo, hi], rewards Bernoulli(0.5)."""
    rng = random.Random(seed)
    out = []
    tid = 0
    for g in range(groups):
        prompt = [rng.randrange(vocab) for _ in range(prompt_len)]
        trajs = []
        for _ in range(per_group):
            if multi_turn:
                turns = []
                for k in range(rng.randint(1, 3)):
                    a = [rng.randrange(vocab) for _ in range(rng.randint(2, 6))]
                    turns.append((a, [True] * len(a)))
                    o = [rng.randrange(vocab) for _ in range(rng.randint(1, 4))]
                    turns.append((o, [False] * len(o)))
                turns.append(([rng.randrange(vocab) for _ in range(3)], [True] * 3))
            else:
                n = rng.randint(lo, hi)
                toks = [rng.randrange(vocab) for _ in range(n)]
                turns = [(toks, [True] * n)]
            trajs.append((tid, turns, float(rng.random() < 0.5)))
            tid += 1
        out.append((g, prompt, trajs))
    order = [(g, t) for g, _, trajs in out for t in trajs]
    rng.shuffle(order)
    return out, order


def advantages(rewards: list[float], eps: float = EPS) -> list[float]:
    r = torch.tensor(rewards, dtype=torch.float64)
    mean, std = float(r.mean()), float(r.std(unbiased=False)) + eps
    return [(x - mean) / std for x in rewards]
