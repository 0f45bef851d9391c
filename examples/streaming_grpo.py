"""Agentic streaming GRPO with this package's trainer: two optimizer steps, no downloads.

Each trajectory is a short agent episode: the model's action (scored tokens)
followed by a tool's reply (unscored tokens), repeated for a few turns. The
episodes of a prompt group finish in a random order; each one is
differentiated the moment its reward arrives (``close_trajectory``), the
group's shared prompt is differentiated once when the group closes, and
``step()`` applies the group-normalised update with the fused flat AdamW.

Run ``python examples/streaming_grpo.py`` (CPU: fp32 torch ops; a B200: bf16
through this package's kernels). For several GPUs launch it with
``torch.distributed.run``; every rank then trains its own groups and the step
averages the gradients across ranks.
"""

import json
import random
import sys
import time
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))
sys.path.insert(1, str(Path(__file__).resolve().parents[1]))  # run from a source checkout

from _tiny_model import VOCAB_SIZE, tiny_qwen3  # noqa: E402

from thundersync_b200.engine.streaming import StreamingRun, arena_for  # noqa: E402
from thundersync_b200.grpo.data_parallel import DataParallelThunderSync  # noqa: E402
from thundersync_b200.parallel.optimizer import FlatAdamW  # noqa: E402

GROUPS, GROUP_SIZE, TURNS = 2, 3, (1, 3)


def episode(rng: random.Random) -> list[tuple[list[int], list[bool]]]:
    """A few (action, tool reply) turns; only the action tokens are scored."""
    turns = []
    for _ in range(rng.randint(*TURNS)):
        action = [rng.randrange(VOCAB_SIZE) for _ in range(rng.randint(3, 8))]
        reply = [rng.randrange(VOCAB_SIZE) for _ in range(rng.randint(2, 6))]
        turns.append((action + reply, [True] * len(action) + [False] * len(reply)))
    return turns


def one_step(trainer, rng: random.Random, step: int) -> dict:
    arrivals = []
    for g in range(GROUPS):
        gid = step * GROUPS + g
        trainer.open_group(gid, [rng.randrange(VOCAB_SIZE) for _ in range(6)])
        tids = [gid * GROUP_SIZE + j for j in range(GROUP_SIZE)]
        trainer.register_group_trajectories(gid, tids)
        arrivals += [(gid, tid, episode(rng), float(rng.random() < 0.5)) for tid in tids]
    rng.shuffle(arrivals)  # episodes finish in any order
    left = {gid: GROUP_SIZE for gid, *_ in arrivals}
    scored = 0
    for gid, tid, turns, reward in arrivals:
        for tokens, mask in turns:
            trainer.append_turn(gid, tid, tokens, mask)
            scored += sum(mask)
        trainer.close_trajectory(tid, reward)  # this episode's backward runs now
        left[gid] -= 1
        if left[gid] == 0:
            trainer.close_group(gid)
    stats = trainer.step()
    return {"scored_tokens": scored, "gradient_norm": float(stats["global_grad_norm"])}


def main():
    torch.manual_seed(7)
    device = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    model = tiny_qwen3(device).train()
    # every trainable parameter is a view into one flat arena; the optimizer updates it in one kernel
    optimizer = FlatAdamW(arena_for(model), lr=1e-5, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0, maximize=True)
    trainer = DataParallelThunderSync.init_from_env(
        model, optimizer, grad_clip=1.0, source_offload_device=None, source_offload_mode="device_resident",
        run_factory=lambda m: StreamingRun(m, boundary_cut=True))
    rng = random.Random(11)
    log = []
    t0 = time.perf_counter()
    for step in range(2):
        log.append(one_step(trainer, rng, step))
    if hasattr(trainer, "shutdown"):
        trainer.shutdown()
    norms = [r["gradient_norm"] for r in log]
    if not all(n > 0 and n == n for n in norms):
        raise RuntimeError(f"expected finite, nonzero gradient norms, got {norms}")
    print(json.dumps({"objective": "grpo", "updates": len(log), "gradient_norm": norms[-1],
                      "scored_tokens": sum(r["scored_tokens"] for r in log),
                      "seconds": round(time.perf_counter() - t0, 3), "device": device.type}))


if __name__ == "__main__":
    main()
