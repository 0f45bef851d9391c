"""One GRPO update from two arriving trajectories; no downloads required."""

import json
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))
# a source checkout works without installing the package
sys.path.insert(1, str(Path(__file__).resolve().parents[1]))

from _tiny_model import tiny_qwen3  # noqa: E402

from thundersync_b200 import RewardLinearBackward, StreamingRun  # noqa: E402


def main():
    torch.manual_seed(7)
    device = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    model = tiny_qwen3(device).train()
    # GRPO increases the advantage-weighted log-probability: the optimizer maximizes.
    optimizer = torch.optim.AdamW(model.parameters(), lr=1e-6, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0,
                                  maximize=True)
    optimizer.zero_grad()
    # boundary_cut: each trajectory's backward stops at the shared prompt,
    # which is backpropagated once when its group closes.
    run = StreamingRun(model, boundary_cut=True)
    objective = RewardLinearBackward(run, model, source_offload_device="cpu")
    objective.open_group(0, [1, 2, 3], [0, 1])
    run.append_turn(0, 0, [4, 5], [True, True])
    objective.close_trajectory(0, 0.0)
    run.append_turn(0, 1, [6, 7, 8], [True, True, True])
    objective.close_trajectory(1, 1.0)
    objective.close_group(0)
    objective.assert_safe_to_step()
    norm = torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
    if not (torch.isfinite(norm) and norm > 0):
        raise RuntimeError(f"expected a finite, nonzero gradient norm, got {float(norm)}")
    optimizer.step()
    print(json.dumps({"objective": "grpo", "updates": 1, "gradient_norm": float(norm)}))


if __name__ == "__main__":
    main()
