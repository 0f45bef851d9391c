"""Exactly-once cross-rank work claims on a compare-and-set key-value store (C40).

Protocol (the interface shared with reference
src/thundersync/scheduling/work_claims.py:1-297, kept so that mixed tooling
reads the same keys): an owner publishes work it has not started -- payload,
then an index entry, then the item's price added to its outstanding ``load``.
Whoever moves the item's claim key from empty to its own rank with one
``compare_set`` runs the item; the store's atomicity gives exactly one
winner. The owner claims each published item right before starting it; a
thief claims first and reads the payload afterwards. An owner writes ``done``
once every item it published is resolved, and a thief stops only when every
peer is done. Keys live under ``<namespace>/<step>/``.

Implementation: every item this rank published has one :class:`_Entry` whose
state moves ``published -> mine`` or ``published -> ceded``; peers' published
items are mirrored in per-peer books that are refreshed incrementally from the
peer's index. Works on any store with ``torch.distributed.Store``'s
``set``/``get``/``add``/``compare_set``/``check``/``delete_key``.
"""

from __future__ import annotations

import enum
import json
import time
from collections import Counter
from collections.abc import Callable, Sequence
from dataclasses import dataclass, field
from typing import Any, Protocol

__all__ = ["ClaimStore", "Offer", "StoreWorkClaims", "WorkClaimError"]


class WorkClaimError(RuntimeError):
    """A caller broke the claim protocol's order."""


class ClaimStore(Protocol):
    def set(self, key: str, value: bytes | str) -> None: ...
    def get(self, key: str) -> bytes: ...
    def add(self, key: str, amount: int) -> int: ...
    def compare_set(self, key: str, expected_value: bytes | str, desired_value: bytes | str) -> bytes: ...
    def check(self, keys: list[str]) -> bool: ...
    def delete_key(self, key: str) -> bool: ...


@dataclass(frozen=True)
class Offer:
    """A peer's published item as a thief sees it."""

    owner: int
    item: int
    price: int


class _State(enum.Enum):
    PUBLISHED = "published"
    MINE = "mine"  # the owner won its own claim
    CEDED = "ceded"  # a thief won it


@dataclass
class _Entry:
    price: int
    state: _State = _State.PUBLISHED


@dataclass
class _PeerBook:
    read_upto: int = 0  # index entries already mirrored
    items: dict[int, Offer] = field(default_factory=dict)


class _Keys:
    """The key scheme: ``<ns>/<step>/<rank>/{payload/<item>, offer/<idx>, offers, load, done}`` and
    ``<ns>/<step>/claim/<item>``."""

    def __init__(self, namespace: str, step: int) -> None:
        self.base = f"{namespace}/{step}"

    def payload(self, owner: int, item: int) -> str:
        return f"{self.base}/{owner}/payload/{item}"

    def index_entry(self, owner: int, idx: int) -> str:
        return f"{self.base}/{owner}/offer/{idx}"

    def index_len(self, owner: int) -> str:
        return f"{self.base}/{owner}/offers"

    def load(self, owner: int) -> str:
        return f"{self.base}/{owner}/load"

    def done(self, owner: int) -> str:
        return f"{self.base}/{owner}/done"

    def claim(self, item: int) -> str:
        return f"{self.base}/claim/{item}"


class StoreWorkClaims:
    """This rank's side of one step's claims (owner of its own items, thief of its peers')."""

    def __init__(self, store: ClaimStore, *, rank: int, world_size: int, namespace: str = "work-claims",
                 clock: Callable[[], float] = time.perf_counter) -> None:
        if world_size < 1 or not 0 <= rank < world_size:
            raise ValueError(f"rank {rank} outside world size {world_size}")
        if not namespace or "/" in namespace:
            raise ValueError(f"namespace {namespace!r} must be a single non-empty key segment")
        self._store = store
        self.rank, self.world_size = int(rank), int(world_size)
        self._namespace = namespace
        self._clock = clock
        self._keys: _Keys | None = None
        self._step: int | None = None
        self._done = False
        self._mine: dict[int, _Entry] = {}
        self._books: dict[int, _PeerBook] = {}
        self._stats: Counter = Counter()

    # ---------------------------------------------------------------- step
    def begin_step(self, step: int) -> None:
        """Start a new step; the previous one must have published ``done``."""
        if self._step is not None and not self._done:
            raise WorkClaimError(f"cannot begin a step: step {self._step} never published done")
        self._step, self._done = int(step), False
        self._keys = _Keys(self._namespace, self._step)
        self._mine = {}
        self._books = {p: _PeerBook() for p in self.peers}
        self._stats = Counter()

    @property
    def step(self) -> int | None:
        return self._step

    @property
    def peers(self) -> list[int]:
        return [r for r in range(self.world_size) if r != self.rank]

    @property
    def done(self) -> bool:
        return self._done

    def _k(self) -> _Keys:
        if self._keys is None:
            raise WorkClaimError("begin_step has not been called")
        return self._keys

    # ---------------------------------------------------------------- owner side
    def offer(self, item: int, price: int, payload: bytes) -> None:
        """Publish an unstarted item: payload, index entry, then its price onto this rank's load."""
        if self._done:
            raise WorkClaimError(f"rank {self.rank} already published done for step {self._step}")
        if item in self._mine:
            raise WorkClaimError(f"item {item} was published twice")
        if price < 0:
            raise ValueError(f"price {price} is negative")
        k = self._k()
        idx = len(self._mine)
        self._store.set(k.payload(self.rank, item), payload)
        self._store.set(k.index_entry(self.rank, idx), json.dumps({"item": int(item), "price": int(price)}))
        self._store.add(k.index_len(self.rank), 1)
        self._store.add(k.load(self.rank), int(price))
        self._mine[item] = _Entry(int(price))
        self._stats.update(offered=1, offered_price=int(price), payload_bytes_out=len(payload))

    def is_offered(self, item: int) -> bool:
        return item in self._mine

    def claim_own(self, items: Sequence[int]) -> tuple[list[int], list[int]]:
        """Claim each item before starting it. Items never published are trivially this rank's.
        Returns (items to run here, items a thief took)."""
        run_here, taken = [], []
        for item in items:
            entry = self._mine.get(item)
            if entry is None:
                run_here.append(item)
                continue
            if entry.state is not _State.PUBLISHED:
                raise WorkClaimError(f"item {item} was already resolved ({entry.state.value})")
            if self._try_claim(item):
                entry.state = _State.MINE
                self._store.delete_key(self._k().payload(self.rank, item))
                self._stats.update(own_claims=1)
                run_here.append(item)
            else:
                entry.state = _State.CEDED
                self._stats.update(ceded=1, ceded_price=entry.price)
                taken.append(item)
        return run_here, taken

    def finish_own(self, items: Sequence[int]) -> None:
        """Take the prices of finished, self-claimed items off this rank's load."""
        settled = 0
        for item in items:
            entry = self._mine.get(item)
            if entry is None:
                continue
            if entry.state is not _State.MINE:
                raise WorkClaimError(f"item {item} is {entry.state.value}, not claimed by its owner")
            settled += entry.price
        if settled:
            self._store.add(self._k().load(self.rank), -settled)

    def publish_done(self) -> None:
        """Declare that this rank publishes nothing more and has resolved everything it published."""
        open_items = sorted(i for i, e in self._mine.items() if e.state is _State.PUBLISHED)
        if open_items:
            raise WorkClaimError(f"cannot publish done: published items {open_items} were never claimed")
        self._store.set(self._k().done(self.rank), "1")
        self._done = True

    # ---------------------------------------------------------------- thief side
    def peer_done(self, peer: int) -> bool:
        return bool(self._store.check([self._k().done(peer)]))

    def all_peers_done(self) -> bool:
        return all(self.peer_done(p) for p in self.peers)

    def peer_load(self, peer: int) -> int:
        return int(self._store.add(self._k().load(peer), 0))

    def open_offers(self, peer: int) -> list[Offer]:
        """The peer's published items nobody has claimed yet (as far as the store shows now)."""
        k = self._k()
        book = self._books[peer]
        listed = int(self._store.add(k.index_len(peer), 0))
        while book.read_upto < listed:
            rec = json.loads(self._store.get(k.index_entry(peer, book.read_upto)))
            book.items[int(rec["item"])] = Offer(peer, int(rec["item"]), int(rec["price"]))
            book.read_upto += 1
        claimed = [item for item in book.items if self._store.check([k.claim(item)])]
        for item in claimed:
            del book.items[item]
        return list(book.items.values())

    def steal(self, offer: Offer) -> bytes | None:
        """Claim a peer's item; on success move its price off the peer's load and return its payload."""
        self._books[offer.owner].items.pop(offer.item, None)
        if not self._try_claim(offer.item):
            return None
        k = self._k()
        self._store.add(k.load(offer.owner), -offer.price)
        payload = self._store.get(k.payload(offer.owner, offer.item))
        self._store.delete_key(k.payload(offer.owner, offer.item))
        self._stats.update(stolen=1, stolen_price=offer.price, payload_bytes_in=len(payload))
        return payload

    # ---------------------------------------------------------------- shared
    def _try_claim(self, item: int) -> bool:
        me = str(self.rank).encode()
        t0 = self._clock()
        holder = self._store.compare_set(self._k().claim(item), "", me)
        self._stats["claim_attempts"] += 1
        self._stats["claim_s"] += self._clock() - t0
        return (holder.encode() if isinstance(holder, str) else bytes(holder)) == me

    _REPORTED = ("offered", "offered_price", "own_claims", "ceded", "ceded_price", "stolen", "stolen_price",
                 "claim_attempts", "claim_s", "payload_bytes_out", "payload_bytes_in")

    def report(self) -> dict[str, Any]:
        out: dict[str, Any] = {"step": self._step, "rank": self.rank, "world_size": self.world_size,
                               "done": self._done}
        out.update({name: self._stats.get(name, 0) for name in self._REPORTED})
        return out
