"""Host-side scheduling: packing, pricing, claims store races, admission, final forest."""

from __future__ import annotations

import threading
from dataclasses import dataclass

import pytest
import torch

from thundersync_b200.grpo.claims import decode_final_work, encode_final_work
from thundersync_b200.grpo.packing import pack_groups
from thundersync_b200.grpo.work_price import attention_weight, lpt_assign, trajectory_price
from thundersync_b200.scheduling.admission import ContentReadyAdmission
from thundersync_b200.scheduling.work_claims import StoreWorkClaims, WorkClaimError


class DictStore:
    """Thread-safe in-memory stand-in for torch.distributed.Store."""

    def __init__(self):
        self.d: dict[str, bytes] = {}
        self.lock = threading.Lock()

    def set(self, k, v):
        with self.lock:
            self.d[k] = v.encode() if isinstance(v, str) else bytes(v)

    def get(self, k):
        with self.lock:
            return self.d[k]

    def add(self, k, n):
        with self.lock:
            v = int(self.d.get(k, b"0")) + n
            self.d[k] = str(v).encode()
            return v

    def compare_set(self, k, exp, want):
        exp = exp.encode() if isinstance(exp, str) else exp
        want = want.encode() if isinstance(want, str) else want
        with self.lock:
            cur = self.d.get(k)
            if cur is None and exp == b"":
                self.d[k] = want
                return want
            if cur == exp:
                self.d[k] = want
                return want
            return cur if cur is not None else exp

    def check(self, keys):
        with self.lock:
            return all(k in self.d for k in keys)

    def delete_key(self, k):
        with self.lock:
            return self.d.pop(k, None) is not None


@dataclass
class Item:
    group_id: int
    traj_id: int
    n_tokens: int


def test_pack_groups_keeps_groups_whole_and_splits_oversized():
    items = [Item(g, t, 10 * (t % 3 + 1)) for g in range(3) for t in range(g * 4, g * 4 + 4)]
    mbs = pack_groups(items, max_tokens_per_microbatch=100)
    for mb in mbs:
        assert len({i.group_id for i in mb}) >= 1
    assert sum(len(mb) for mb in mbs) == len(items)
    big = [Item(0, t, 60) for t in range(3)]
    mbs = pack_groups(big, max_tokens_per_microbatch=100, split_oversized_groups=True)
    assert [len(m) for m in mbs] == [1, 1, 1]
    with pytest.raises(ValueError):
        pack_groups(items, max_tokens_per_microbatch=0)


def test_price_and_lpt():
    class C:
        num_hidden_layers, num_attention_heads, head_dim, hidden_size = 2, 4, 16, 64

    w = attention_weight(C, 1000)
    assert w == pytest.approx(2 * 4 * 16 / 1000)
    assert trajectory_price(10, 5, 0.0) == 5
    assert trajectory_price(10, 5, 1.0) == 5 + 15 * 15 - 100
    place = lpt_assign([(1, 10), (2, 9), (3, 1), (4, 1)], 2)
    assert place[1] != place[2]
    assert lpt_assign([(1, 10), (2, 9), (3, 1), (4, 1)], 2) == place


def test_payload_roundtrip_is_exact():
    adv = 1 / 3
    p = encode_final_work(group_id=2, trajectory_id=7, advantage=adv, prompt_tokens=[1, 2],
                          turns=[([3, 4], [True, False])])
    g, t, a, pr, turns = decode_final_work(p)
    assert (g, t, pr, turns) == (2, 7, [1, 2], [([3, 4], [True, False])]) and a == adv


def test_claims_exactly_once_under_races():
    store = DictStore()
    world = 4
    views = [StoreWorkClaims(store, rank=r, world_size=world) for r in range(world)]
    for v in views:
        v.begin_step(1)
    owner = views[0]
    for item in range(200):
        owner.offer(item, 1 + item % 5, f"payload-{item}".encode())
    winners: dict[int, list[int]] = {}
    lock = threading.Lock()

    def thief(v):
        for peer in v.peers:
            for offer in v.open_offers(peer):
                if v.steal(offer) is not None:
                    with lock:
                        winners.setdefault(offer.item, []).append(v.rank)

    threads = [threading.Thread(target=thief, args=(v,)) for v in views[1:]]
    for t in threads:
        t.start()
    won, lost = owner.claim_own(list(range(200)))
    for t in threads:
        t.join()
    for item in won:
        winners.setdefault(item, []).append(0)
    assert sorted(winners) == list(range(200))
    assert all(len(v) == 1 for v in winners.values())
    assert set(lost) == {i for i, r in winners.items() if r[0] != 0}
    owner.finish_own(won)
    owner.publish_done()
    with pytest.raises(WorkClaimError):
        owner.offer(999, 1, b"x")


class FakeTrainer:
    def __init__(self):
        self.calls = []
        self.closed = set()

    def prepare_trajectories(self, ids):
        self.calls.append(("prepare", tuple(ids)))

    def bind_rewards(self, binds):
        self.calls.append(("bind", tuple(binds)))

    def close_trajectories(self, closes):
        self.calls.append(("close", tuple(closes)))

    def close_group(self, gid):
        self.calls.append(("group", gid))

    def group_reduction_complete(self, gid):
        return True


def test_content_ready_admission_flow():
    tr = FakeTrainer()
    adm = ContentReadyAdmission(tr, group_size=2, max_prepare_pack=2)
    adm.add_completion(0, 10)
    adm.add_completion(0, 11)
    adm.flush_prepares()
    assert tr.calls == [("prepare", (10, 11))]
    adm.bind_verdict(0, 10, 1.0)
    adm.bind_verdict(0, 11, 0.0)
    adm.close_ready_groups()
    assert tr.calls[-1] == ("group", 0)
    adm.drain_group_closes()


def _ids(mbs):
    return [[i.traj_id for i in mb] for mb in mbs]


def test_pack_groups_orders_groups_and_members_and_flushes_before_a_split():
    # groups arrive out of order; whole groups pack greedily in group order under the budget
    items = [Item(2, 21, 5), Item(0, 1, 4), Item(1, 11, 3), Item(0, 0, 4), Item(2, 20, 5), Item(1, 10, 3)]
    assert _ids(pack_groups(items, max_tokens_per_microbatch=14)) == [[0, 1, 10, 11], [20, 21]]
    # an oversized group stays whole unless splitting is asked for
    big = [Item(0, 0, 2), Item(1, 10, 7), Item(1, 11, 7), Item(1, 12, 7), Item(2, 20, 1)]
    assert _ids(pack_groups(big, max_tokens_per_microbatch=10)) == [[0], [10, 11, 12], [20]]
    # with splitting, the open micro-batch flushes first and the group's runs each fit the budget
    assert _ids(pack_groups(big, max_tokens_per_microbatch=10, split_oversized_groups=True)) == [
        [0], [10], [11], [12], [20]]
    assert _ids(pack_groups(big, max_tokens_per_microbatch=14, split_oversized_groups=True)) == [
        [0], [10, 11], [12], [20]]


@pytest.mark.parametrize("split", [False, True])
def test_pack_groups_places_every_trajectory_once_in_canonical_order(split):
    import random

    rng = random.Random(5)
    items = [Item(g, g * 100 + j, rng.randint(1, 9)) for g in rng.sample(range(6), 6) for j in range(rng.randint(1, 5))]
    rng.shuffle(items)
    mbs = pack_groups(items, max_tokens_per_microbatch=12, split_oversized_groups=split)
    flat = [i.traj_id for mb in mbs for i in mb]
    assert flat == sorted(i.traj_id for i in items)
    if split:
        assert all(sum(i.n_tokens for i in mb) <= 12 or len(mb) == 1 for mb in mbs)
