"""Worker of the failure-detection tests: gloo ranks on the CPU, failures injected on the host.

Scenarios (argv[1]):
  heartbeat  rank 2 stops beating (alive but hung), rank 1 exits orderly; rank 0 must
             report both within the timeout.
  pgtimeout  rank 2 dies before a collective; ranks 0 and 1 must get an error from the
             all_reduce within the short process-group timeout instead of hanging.
Rank 0 writes {"dead": [...], "elapsed": s, ...} to argv[2]."""
import json
import os
import sys
import time
from datetime import timedelta

import torch
import torch.distributed as dist

from air_rs.parallel.health import CommTimeout, Heartbeat


def heartbeat(out):
    r, w = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    store = dist.TCPStore("127.0.0.1", int(os.environ["MASTER_PORT"]) + 7, w, r == 0, timeout=timedelta(seconds=30))
    hb = Heartbeat(store, r, w, interval=0.05, timeout=0.6).start()
    store.add("ready", 1)
    while store.add("ready", 0) < w:
        time.sleep(0.01)
    if r == 2:
        hb.pause()
        time.sleep(4.0)
        return
    if r == 1:
        time.sleep(0.3)
        hb.stop(orderly=True)
        time.sleep(4.0)
        return
    t0 = time.monotonic()
    dead = []
    while time.monotonic() - t0 < 3.0:
        dead = hb.dead_ranks()
        if sorted(dead) == [1, 2]:
            break
        time.sleep(0.05)
    raised = False
    try:
        hb.check()
    except CommTimeout:
        raised = True
    json.dump({"dead": sorted(dead), "elapsed": time.monotonic() - t0, "raised": raised}, open(out, "w"))
    hb.stop()


def pgtimeout(out):
    dist.init_process_group("gloo", timeout=timedelta(seconds=3))
    r = dist.get_rank()
    dist.barrier()
    if r == 2:
        os._exit(0)                   # dies without joining the next collective
    t0 = time.monotonic()
    err = None
    try:
        dist.all_reduce(torch.ones(4))
    except Exception as e:
        err = type(e).__name__
    if r == 0:
        json.dump({"error": err, "elapsed": time.monotonic() - t0}, open(out, "w"))
    os._exit(0)


if __name__ == "__main__":
    {"heartbeat": heartbeat, "pgtimeout": pgtimeout}[sys.argv[1]](sys.argv[2])
