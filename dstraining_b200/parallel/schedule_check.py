"""Deadlock check of the pipeline schedules, without running them.

    python -m dstraining_b200.parallel.schedule_check --pp 4 --chunks 2 --micro-batches 8

Builds every rank's sequence of communication events from the same op
orders the schedules execute (:func:`~dstraining_b200.parallel.pipeline.order_1f1b`,
:func:`~dstraining_b200.parallel.pipeline.order_interleaved`) and plays them
against each other. Each directed link (flow ``fwd`` / ``bwd``, source rank,
destination rank) is its own FIFO channel, as the schedules give every link
its own two-rank communicator. Two delivery models:

* ``buffered``: a send never blocks its rank; a receive waits until the
  matching message was sent. This is how the schedules run: sends are
  fire-and-forget and the compute stream waits only on receives.
* ``rendezvous``: a send also waits until the receiver has reached the
  matching receive - the strictest model (a transport with no buffering).

A schedule passes when every rank finishes and every link delivers exactly
the messages its receiver expects. The reference's interleaved schedule
deadlocked on NCCL once TP or DP groups were added (its ``README.md:275-283``);
this check covers the ordering side of that failure for any (p, v, m).
"""

from __future__ import annotations

import argparse
import json
import sys
from collections import defaultdict
from typing import Dict, List, Tuple

from .pipeline import interleaved_chunk, order_1f1b, order_interleaved

Event = Tuple[str, Tuple[str, int, int]]  # ("send" | "recv", (flow, src, dst))


def programs(p: int, v: int, m: int) -> List[List[Event]]:
    """Every rank's communication events in order (``v == 1``: 1F1B on a line
    of stages; ``v > 1``: the interleaved schedule on a ring; one rank has
    none)."""
    progs: List[List[Event]] = []
    if p == 1:
        return [[]]  # one rank: chunks pass activations in memory
    for r in range(p):
        ev: List[Event] = []
        if v == 1:
            for op, _ in order_1f1b(p, r, m):
                if op == "F":
                    if r > 0:
                        ev.append(("recv", ("fwd", r - 1, r)))
                    if r < p - 1:
                        ev.append(("send", ("fwd", r, r + 1)))
                else:
                    if r < p - 1:
                        ev.append(("recv", ("bwd", r + 1, r)))
                    if r > 0:
                        ev.append(("send", ("bwd", r, r - 1)))
        else:
            prev, nxt = (r - 1) % p, (r + 1) % p
            for op, k in order_interleaved(p, r, v, m):
                c = interleaved_chunk(k, p, v, op == "F")
                vfirst, vlast = r == 0 and c == 0, r == p - 1 and c == v - 1
                if op == "F":
                    if not vfirst:
                        ev.append(("recv", ("fwd", prev, r)))
                    if not vlast:
                        ev.append(("send", ("fwd", r, nxt)))
                else:
                    if not vlast:
                        ev.append(("recv", ("bwd", nxt, r)))
                    if not vfirst:
                        ev.append(("send", ("bwd", r, prev)))
        progs.append(ev)
    return progs


def simulate(progs: List[List[Event]], model: str = "buffered") -> Dict:
    """Play the ranks' events against each other; returns ``ok``, the final
    position of every rank and, on a deadlock, what each stuck rank waits for."""
    pc = [0] * len(progs)
    sent: Dict = defaultdict(int)
    received: Dict = defaultdict(int)
    progress = True
    while progress:
        progress = False
        for r, ev in enumerate(progs):
            while pc[r] < len(ev):
                kind, link = ev[pc[r]]
                if kind == "send":
                    if model == "rendezvous":
                        dst = link[2]
                        nxt = progs[dst][pc[dst]] if pc[dst] < len(progs[dst]) else None
                        if nxt != ("recv", link) or received[link] != sent[link]:
                            break
                        received[link] += 1
                        pc[dst] += 1
                    sent[link] += 1
                else:
                    if received[link] >= sent[link]:
                        break
                    received[link] += 1
                pc[r] += 1
                progress = True
    done = all(pc[r] == len(ev) for r, ev in enumerate(progs))
    stuck = {r: progs[r][pc[r]] for r in range(len(progs)) if pc[r] < len(progs[r])}
    undelivered = {str(k): sent[k] - received[k] for k in sent if sent[k] != received[k]}
    return {"ok": done and not undelivered, "positions": pc, "stuck": {r: str(e) for r, e in stuck.items()},
            "undelivered": undelivered}


def check(p: int, v: int, m: int, model: str = "buffered") -> Dict:
    return simulate(programs(p, v, m), model)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="deadlock check of the pipeline schedules")
    ap.add_argument("--pp", type=int, required=True)
    ap.add_argument("--chunks", type=int, default=1)
    ap.add_argument("--micro-batches", type=int, required=True)
    ap.add_argument("--model", choices=["buffered", "rendezvous"], default="buffered")
    a = ap.parse_args(argv)
    if a.chunks > 1 and a.micro_batches % a.pp:
        raise SystemExit("interleaving needs micro-batches divisible by pp")
    out = check(a.pp, a.chunks, a.micro_batches, a.model)
    print(json.dumps(out))
    sys.exit(0 if out["ok"] else 1)


if __name__ == "__main__":
    main()
