"""Exactly-once cross-rank work claims over a compare-and-set key-value store (C40).

An owner *offers* work it has not started (payload first, then an index
entry, then its price joins the owner's outstanding ``load``). Any rank --
the owner included -- *claims* an item by a ``compare_set`` of the item's
claim key from empty to its rank; the store's atomicity makes exactly one
claimant win. The owner claims each offered item before starting it and
skips the ones it lost; a thief steals by the same claim and then reads the
payload. ``done`` is published once the owner has resolved every offer and
will offer no more this step, so a thief may stop only when all peers are
done. All keys are scoped by namespace and step. The protocol is the
reference's (src/thundersync/scheduling/work_claims.py:1-297); this module is
written against ``torch.distributed.Store``'s C++ TCPStore primitives
(``set``/``get``/``add``/``compare_set``/``check``/``delete_key``).
"""

from __future__ import annotations

import json
import time
from collections.abc import Callable, Sequence
from dataclasses import dataclass
from typing import Any, Protocol

__all__ = ["ClaimStore", "Offer", "StoreWorkClaims", "WorkClaimError"]


class WorkClaimError(RuntimeError):
    pass


class ClaimStore(Protocol):
    def set(self, key: str, value: bytes | str) -> None: ...
    def get(self, key: str) -> bytes: ...
    def add(self, key: str, amount: int) -> int: ...
    def compare_set(self, key: str, expected_value: bytes | str, desired_value: bytes | str) -> bytes: ...
    def check(self, keys: list[str]) -> bool: ...
    def delete_key(self, key: str) -> bool: ...


@dataclass(frozen=True)
class Offer:
    owner: int
    item: int
    price: int


_COUNTERS = ("offered", "offered_price", "own_claims", "ceded", "ceded_price", "stolen", "stolen_price",
             "claim_attempts", "claim_s", "payload_bytes_out", "payload_bytes_in")


class StoreWorkClaims:
    """One rank's view of one step's claims."""

    def __init__(self, store: ClaimStore, *, rank: int, world_size: int, namespace: str = "work-claims",
                 clock: Callable[[], float] = time.perf_counter) -> None:
        if world_size < 1 or not 0 <= rank < world_size:
            raise ValueError(f"rank {rank} is not in a world of {world_size}")
        if not namespace or "/" in namespace:
            raise ValueError("the namespace must be one nonempty key segment")
        self._store = store
        self.rank, self.world_size = int(rank), int(world_size)
        self._ns = namespace
        self._clock = clock
        self._step: int | None = None
        self._done = False
        self._offered: dict[int, int] = {}
        self._n_offers = 0
        self._mine: set[int] = set()
        self._lost: set[int] = set()
        self._cursor: dict[int, int] = {}
        self._open: dict[int, dict[int, Offer]] = {}
        self._c: dict[str, float] = {}

    # keys -------------------------------------------------------------
    def _k(self, *parts: object) -> str:
        if self._step is None:
            raise WorkClaimError("no step has begun")
        return "/".join([self._ns, str(self._step), *map(str, parts)])

    # step -------------------------------------------------------------
    def begin_step(self, step: int) -> None:
        if self._step is not None and not self._done:
            raise WorkClaimError(f"step {self._step} ended without publishing done")
        self._step = int(step)
        self._done = False
        self._offered, self._n_offers = {}, 0
        self._mine, self._lost = set(), set()
        self._cursor = {p: 0 for p in self.peers}
        self._open = {p: {} for p in self.peers}
        self._c = dict.fromkeys(_COUNTERS, 0)

    @property
    def step(self) -> int | None:
        return self._step

    @property
    def peers(self) -> list[int]:
        return [r for r in range(self.world_size) if r != self.rank]

    @property
    def done(self) -> bool:
        return self._done

    # owner ------------------------------------------------------------
    def offer(self, item: int, price: int, payload: bytes) -> None:
        if self._done:
            raise WorkClaimError("an owner that is done offers nothing more")
        if item in self._offered:
            raise WorkClaimError(f"item {item} is already offered")
        if price < 0:
            raise ValueError("an offer's price must not be negative")
        self._store.set(self._k(self.rank, "payload", item), payload)
        self._store.set(self._k(self.rank, "offer", self._n_offers), json.dumps({"item": int(item), "price": int(price)}))
        self._n_offers += 1
        self._store.add(self._k(self.rank, "offers"), 1)
        self._store.add(self._k(self.rank, "load"), int(price))
        self._offered[item] = int(price)
        self._c["offered"] += 1
        self._c["offered_price"] += int(price)
        self._c["payload_bytes_out"] += len(payload)

    def is_offered(self, item: int) -> bool:
        return item in self._offered

    def claim_own(self, items: Sequence[int]) -> tuple[list[int], list[int]]:
        won, lost = [], []
        for item in items:
            if item not in self._offered:
                won.append(item)
                continue
            if item in self._mine:
                raise WorkClaimError(f"item {item} is already claimed by its owner")
            if self._cas(item):
                self._mine.add(item)
                self._c["own_claims"] += 1
                self._store.delete_key(self._k(self.rank, "payload", item))
                won.append(item)
            else:
                self._lost.add(item)
                self._c["ceded"] += 1
                self._c["ceded_price"] += self._offered[item]
                lost.append(item)
        return won, lost

    def finish_own(self, items: Sequence[int]) -> None:
        total = 0
        for item in items:
            if item not in self._offered:
                continue
            if item not in self._mine:
                raise WorkClaimError(f"item {item} was not claimed by its owner")
            total += self._offered[item]
        if total:
            self._store.add(self._k(self.rank, "load"), -total)

    def publish_done(self) -> None:
        pending = set(self._offered) - self._mine - self._lost
        if pending:
            raise WorkClaimError(f"items {sorted(pending)} are offered and unresolved; claim them before publishing done")
        self._store.set(self._k(self.rank, "done"), "1")
        self._done = True

    # thief ------------------------------------------------------------
    def peer_done(self, peer: int) -> bool:
        return bool(self._store.check([self._k(peer, "done")]))

    def all_peers_done(self) -> bool:
        return all(self.peer_done(p) for p in self.peers)

    def peer_load(self, peer: int) -> int:
        return int(self._store.add(self._k(peer, "load"), 0))

    def open_offers(self, peer: int) -> list[Offer]:
        listed = int(self._store.add(self._k(peer, "offers"), 0))
        book = self._open[peer]
        for idx in range(self._cursor[peer], listed):
            e = json.loads(self._store.get(self._k(peer, "offer", idx)))
            book[int(e["item"])] = Offer(peer, int(e["item"]), int(e["price"]))
        self._cursor[peer] = listed
        for item in list(book):
            if self._store.check([self._k("claim", item)]):
                del book[item]
        return list(book.values())

    def steal(self, offer: Offer) -> bytes | None:
        self._open[offer.owner].pop(offer.item, None)
        if not self._cas(offer.item):
            return None
        self._store.add(self._k(offer.owner, "load"), -offer.price)
        key = self._k(offer.owner, "payload", offer.item)
        payload = self._store.get(key)
        self._store.delete_key(key)
        self._c["stolen"] += 1
        self._c["stolen_price"] += offer.price
        self._c["payload_bytes_in"] += len(payload)
        return payload

    # shared -----------------------------------------------------------
    def _cas(self, item: int) -> bool:
        t0 = self._clock()
        me = str(self.rank).encode()
        holder = self._store.compare_set(self._k("claim", item), "", me)
        self._c["claim_attempts"] += 1
        self._c["claim_s"] += self._clock() - t0
        if isinstance(holder, str):
            holder = holder.encode()
        return bytes(holder) == me

    def report(self) -> dict[str, Any]:
        return {"step": self._step, "rank": self.rank, "world_size": self.world_size, "done": self._done, **self._c}
