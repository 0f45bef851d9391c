"""On-policy distillation with per-action teacher scores: one update over two episodes.

An episode alternates the student's actions (scored tokens) with observations
(unscored). A teacher scores each action as soon as it exists; the student's
backward for that action runs at once (``append_scored_turn``), and the
adjoint that later actions send back into earlier turns is replayed when the
episode closes (``turn_boundary_rebuild``). The loss is the token-mean of
``ratio · (old − teacher)`` over the batch's scored tokens, so the optimizer
minimises. The teacher here is synthetic: scores drawn from −Exponential(1.5),
clipped to [−20, 0].

Run ``python examples/streaming_opd.py`` (CPU fp32, or bf16 on a B200).
"""

import json
import random
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))
sys.path.insert(1, str(Path(__file__).resolve().parents[1]))  # run from a source checkout

from _tiny_model import VOCAB_SIZE, tiny_qwen3  # noqa: E402

from thundersync_b200 import OPDTurnStream, StreamingRun  # noqa: E402


def teacher_scores(rng: random.Random, n: int, device: torch.device) -> torch.Tensor:
    return torch.tensor([max(-20.0, -rng.expovariate(1 / 1.5)) for _ in range(n)], device=device)


def main():
    torch.manual_seed(3)
    device = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    model = tiny_qwen3(device).eval()  # replay at close needs the same forward as at arrival
    optimizer = torch.optim.AdamW(model.parameters(), lr=1e-6, weight_decay=0.0)
    optimizer.zero_grad()
    run = StreamingRun(model, boundary_cut=True, stream_turns=True, turn_boundary_rebuild=True)
    objective = OPDTurnStream(run, model)
    rng = random.Random(5)
    objective.open_group(0, [rng.randrange(VOCAB_SIZE) for _ in range(5)])
    actions = 0
    for episode in (0, 1):
        for _ in range(rng.randint(2, 3)):
            obs = [rng.randrange(VOCAB_SIZE) for _ in range(rng.randint(1, 4))]
            act = [rng.randrange(VOCAB_SIZE) for _ in range(rng.randint(2, 5))]
            mask = [False] * len(obs) + [True] * len(act)
            objective.append_scored_turn(0, episode, obs + act, mask,
                                         teacher_logprobs=teacher_scores(rng, len(act), device))
            actions += 1
        objective.close_trajectory(episode)  # replays this episode's deferred turn adjoints
    objective.close_group(0)
    objective.assert_safe_to_step()
    norm = float(torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0))
    if not (norm > 0 and norm == norm):
        raise RuntimeError(f"expected a finite, nonzero gradient norm, got {norm}")
    optimizer.step()
    print(json.dumps({"objective": "opd", "updates": 1, "gradient_norm": norm, "actions": actions,
                      "loss": objective.loss_value, "device": device.type}))


if __name__ == "__main__":
    main()
