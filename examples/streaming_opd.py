"""One on-policy-distillation update from a two-turn trajectory; no downloads required."""

import json
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))
# a source checkout works without installing the package
sys.path.insert(1, str(Path(__file__).resolve().parents[1]))

from _tiny_model import tiny_qwen3  # noqa: E402

from thundersync_b200 import OPDTurnStream, StreamingRun  # noqa: E402


def main():
    torch.manual_seed(7)
    device = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    # Turn replay requires a deterministic forward: eval mode.
    model = tiny_qwen3(device).eval()
    # OPD decreases a divergence from the teacher: the optimizer minimizes.
    optimizer = torch.optim.AdamW(model.parameters(), lr=1e-6, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0)
    optimizer.zero_grad()
    # stream_turns: each turn is forwarded on arrival so its teacher-scored
    # loss backwards at once; turn_boundary_rebuild: each turn's outgoing
    # state is cut and replayed in reverse when the trajectory closes.
    run = StreamingRun(model, boundary_cut=True, stream_turns=True, turn_boundary_rebuild=True)
    objective = OPDTurnStream(run, model)
    objective.open_group(0, [1, 2, 3])
    # Teacher log-probabilities for exactly the generated (True) tokens.
    objective.append_scored_turn(0, 0, [4, 5], [True, True],
                                 teacher_logprobs=torch.tensor([-1.5, -1.2], device=device))
    if not any(p.grad is not None and bool(p.grad.abs().sum()) for p in model.parameters()):
        raise RuntimeError("the first scored turn produced no gradient")
    objective.append_scored_turn(0, 0, [6, 7, 8], [False, True, True],
                                 teacher_logprobs=torch.tensor([-1.4, -1.1], device=device))
    objective.close_trajectory(0)
    objective.close_group(0)
    objective.assert_safe_to_step()
    norm = torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
    if not (torch.isfinite(norm) and norm > 0):
        raise RuntimeError(f"expected a finite, nonzero gradient norm, got {float(norm)}")
    optimizer.step()
    print(json.dumps({"objective": "opd", "updates": 1, "gradient_norm": float(norm)}))


if __name__ == "__main__":
    main()
