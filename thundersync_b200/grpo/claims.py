"""Final-work claims for GRPO: any rank may run another rank's final trajectories (C41).

A *final* trajectory (every reward of its group landed, so its float64
advantage is known) is offered with a self-contained payload: group id,
trajectory id, the advantage's exact float64 bits, prompt and turns. The
owner claims each chunk before running it and cedes what a thief won; an idle
rank steals from the peer with the most outstanding work, largest price
first, taking an offer only while what it takes stays at most half the
owner's remaining load. Payload schema and rules match reference
src/thundersync/grpo/claims.py:51-426.
"""

from __future__ import annotations

import json
import time
from collections.abc import Callable, Sequence
from typing import Any, Protocol

from thundersync_b200.grpo.admission import FinalFirstAdmission, GroupLedgerTrainer
from thundersync_b200.scheduling.admission import Close
from thundersync_b200.scheduling.admission import CloseCoefficient, TrainerCall, direct_call
from thundersync_b200.scheduling.work_claims import Offer, StoreWorkClaims

__all__ = ["PAYLOAD_SCHEMA", "ClaimTrainer", "ClaimingFinalFirstAdmission", "decode_final_work", "encode_final_work"]

PAYLOAD_SCHEMA = "thundersync-final-work-v1"


def encode_final_work(*, group_id: int, trajectory_id: int, advantage: float, prompt_tokens: Sequence[int],
                      turns: Sequence[tuple[Sequence[int], Sequence[bool]]]) -> bytes:
    record = {
        "schema": PAYLOAD_SCHEMA,
        "group_id": int(group_id),
        "trajectory_id": int(trajectory_id),
        "advantage": float(advantage).hex(),
        "prompt_tokens": [int(t) for t in prompt_tokens],
        "turns": [[[int(t) for t in tokens], "".join("1" if s else "0" for s in scored)] for tokens, scored in turns],
    }
    return json.dumps(record, separators=(",", ":")).encode()


def decode_final_work(payload: bytes) -> tuple[int, int, float, list[int], list[tuple[list[int], list[bool]]]]:
    rec = json.loads(payload)
    if rec.get("schema") != PAYLOAD_SCHEMA:
        raise ValueError(f"final work payload schema {rec.get('schema')!r} differs")
    turns = [([int(t) for t in tk], [c == "1" for c in sc]) for tk, sc in rec["turns"]]
    return (int(rec["group_id"]), int(rec["trajectory_id"]), float.fromhex(rec["advantage"]),
            [int(t) for t in rec["prompt_tokens"]], turns)


class ClaimTrainer(GroupLedgerTrainer, Protocol):
    def final_work(self, trajectory_id: int) -> tuple[int, int, bytes]: ...
    def cede_final_closes(self, closes: list[tuple[int, CloseCoefficient]]) -> None: ...
    def run_claimed_work(self, payloads: list[bytes]) -> None: ...
    def record_work_claims(self, report: dict[str, Any]) -> None: ...

    @property
    def final_forest_max_tokens(self) -> int: ...


class ClaimingFinalFirstAdmission(FinalFirstAdmission):
    def __init__(self, trainer: ClaimTrainer, *, group_size: int, trainer_call: TrainerCall = direct_call,
                 claims: StoreWorkClaims, poll_s: float = 0.02, timeout_s: float = 3600.0,
                 sleep: Callable[[float], None] = time.sleep, clock: Callable[[], float] = time.monotonic,
                 **options: Any) -> None:
        if not options.get("final_forest"):
            raise ValueError("claiming final work needs the final forest")
        super().__init__(trainer, group_size=group_size, trainer_call=trainer_call, **options)
        if poll_s <= 0 or timeout_s < 0:
            raise ValueError("poll_s must be positive and timeout_s nonnegative")
        self._ct = trainer
        self._claims = claims
        self._poll_s, self._timeout_s = float(poll_s), float(timeout_s)
        self._sleep, self._clock = sleep, clock
        self._sizes: dict[int, tuple[int, int]] = {}
        self._idle_polls = 0
        self._idle_s = 0.0
        claims.begin_step((claims.step or 0) + 1)

    # owner --------------------------------------------------------------
    def _offer_final_work(self) -> None:
        for c in self._closes:
            if not self._is_final(c.group) or self._claims.is_offered(c.trajectory):
                continue
            tokens, price, payload = self._ct.final_work(c.trajectory)
            self._sizes[c.trajectory] = (tokens, price)
            self._claims.offer(c.trajectory, price, payload)

    def drain_ready_closes(self) -> None:
        self._offer_final_work()
        super().drain_ready_closes()

    @property
    def deferred_work_reason(self) -> str | None:
        r = super().deferred_work_reason
        if r is not None:
            return r
        return None if self._claims.all_peers_done() else "peer_work"

    def close_ready_groups(self) -> None:
        super().close_ready_groups()
        if FinalFirstAdmission.deferred_work_reason.fget(self) is None and not self._events_pending():
            self._claim_peer_batch()

    def _claim(self, chunk: list[Close]) -> list[Close]:
        """Claim our own offered closes; hand the ones a peer took to the trainer as ceded."""
        won_ids, lost_ids = self._claims.claim_own([c.trajectory for c in chunk])
        lost = set(lost_ids)
        if lost:
            ceded = [c for c in chunk if c.trajectory in lost]
            self._ct.cede_final_closes([(c.trajectory, c.coefficient) for c in ceded])
            for c in ceded:
                self._mark_bound(c.group)
        won = set(won_ids)
        return [c for c in chunk if c.trajectory in won]

    def _final_forest(self, closes: list[Close]) -> None:
        cap = self._ct.final_forest_max_tokens
        queue = list(closes)
        while queue:
            chunk, tokens = [], 0
            while queue:
                size = self._sizes.get(queue[0].trajectory, (0, 0))[0]
                if chunk and tokens + size > cap:
                    break
                chunk.append(queue.pop(0))
                tokens += size
            won = self._claim(chunk)
            if won:
                super()._final_forest(won)
                self._claims.finish_own([c.trajectory for c in won])
            if queue and self._interrupted():
                self._closes = queue + self._closes
                return

    def _drain(self, closes: list[Close], *, gated: bool, **labels: Any) -> list[Close]:
        if labels.get("job_class") != "final":
            return super()._drain(closes, gated=gated, **labels)
        rest = list(closes)
        size = self._pack_size(len(rest))
        while rest:
            chunk, rest = rest[:size], rest[size:]
            won = self._claim(chunk)
            if won:
                super()._drain(won, gated=gated, **labels)
                self._claims.finish_own([c.trajectory for c in won])
        return []

    # step end -------------------------------------------------------------
    def drain_group_closes(self) -> None:
        super().drain_group_closes()
        self._claims.publish_done()
        self._claim_peer_work()
        self._ct.record_work_claims({**self._claims.report(), "idle_polls": self._idle_polls, "idle_s": self._idle_s})

    def _claim_peer_work(self) -> None:
        deadline = self._clock() + self._timeout_s if self._timeout_s else None
        while not self._claims.all_peers_done():
            if not self._claim_peer_batch():
                if deadline is not None and self._clock() > deadline:
                    raise RuntimeError(f"work claims: peers did not finish their step within {self._timeout_s:.0f} s")
                self._idle_polls += 1
                t0 = self._clock()
                self._sleep(self._poll_s)
                self._idle_s += self._clock() - t0

    def _claim_peer_batch(self) -> bool:
        batch = self._steal_batch()
        if not batch:
            return False
        payloads, got = [], []
        for offer in batch:
            p = self._claims.steal(offer)
            if p is not None:
                payloads.append(p)
                got.append(offer)
        if payloads:
            self._call("trajectory_backward", lambda p=payloads: self._ct.run_claimed_work(p),
                       trajectory_count=len(got), trajectory_ids=[o.item for o in got],
                       owner_ranks=sorted({o.owner for o in got}), job_class="claimed")
        return True

    def _steal_batch(self) -> list[Offer]:
        best = None
        for peer in self._claims.peers:
            if self._claims.peer_done(peer):
                continue
            load = self._claims.peer_load(peer)
            if best is None or load > best[1]:
                best = (peer, load)
        if best is None or best[1] <= 0:
            return []
        peer, load = best
        cap = self._ct.final_forest_max_tokens
        taken, out = 0, []
        for offer in sorted(self._claims.open_offers(peer), key=lambda o: (-o.price, o.item)):
            if out and taken + offer.price > cap:
                continue
            if 2 * (taken + offer.price) > load:
                continue
            out.append(offer)
            taken += offer.price
        return out
