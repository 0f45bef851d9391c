"""torchrun worker for tests/test_claims_gloo.py (CPU; not collected by pytest).

Four processes share the process group's TCPStore. Rank 0 offers 500 items and claims its own list
while the other ranks steal whatever is still offered; every item must end with exactly one winner.
Then the claiming-admission steps run three times with a barrier between them.
"""

from __future__ import annotations

import argparse
import datetime
import json
import sys
from pathlib import Path

import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from thundersync_b200.scheduling.work_claims import StoreWorkClaims  # noqa: E402

ITEMS = 500


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    args = ap.parse_args()
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    rank, world = dist.get_rank(), dist.get_world_size()
    store = dist.distributed_c10d._get_default_store()
    report = []
    for step in range(1, 4):
        claims = StoreWorkClaims(store, rank=rank, world_size=world, namespace=f"race-{step}")
        claims.begin_step(step)
        if rank == 0:
            for item in range(ITEMS):
                claims.offer(item, 1 + item % 7, f"payload-{item}".encode())
        dist.barrier()
        won: list[int] = []
        if rank == 0:
            won, _lost = claims.claim_own(list(range(ITEMS)))
            claims.finish_own(won)
        else:
            for offer in claims.open_offers(0):
                if claims.steal(offer) is not None:
                    won.append(offer.item)
        claims.publish_done()
        dist.barrier()
        everyone = [None] * world
        dist.all_gather_object(everyone, won)
        report.append(everyone)
        dist.barrier()
    if rank == 0:
        Path(args.out).write_text(json.dumps(report))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
