"""Worker for the failure-detection tests (one process per rank, gloo). Modes:
leave  : rank 1 stops heartbeating and exits between steps; rank 0 must stop at its next step boundary with
         PeerFailure instead of entering the next collective.
raise  : rank 1 raises during a step; rank 0's next collective must end with an error within the short
         process-group timeout."""
import datetime
import os
import sys
import time

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from arcagi2_flashnext_dots3_b200.utils.failure import Heartbeat, PeerFailure, StepGuard  # noqa: E402


def main():
    mode = sys.argv[1]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=4))
    store = dist.distributed_c10d._get_default_store()
    hb = Heartbeat(store, rank, world, period=0.1, limit=1.0).start()
    x = torch.ones(4)
    for step in range(200):
        if mode == "raise" and rank == 1 and step == 3:
            raise RuntimeError("injected failure on rank 1")
        try:
            with StepGuard(hb):
                dist.all_reduce(x)
        except PeerFailure as e:
            print(f"RANK{rank}_DETECTED_PEER_FAILURE step={step} {e}", flush=True)
            os._exit(0)
        except Exception as e:  # collective failed because a peer is gone
            print(f"RANK{rank}_COLLECTIVE_ERROR step={step} {type(e).__name__}", flush=True)
            os._exit(0)
        if mode == "leave" and rank == 1 and step == 2:
            hb.stop()
            os._exit(0)  # leaves right after a completed step: nothing in flight
        time.sleep(0.05 if mode == "raise" else 1.5)  # host work between steps longer than the limit
    print(f"RANK{rank}_NO_DETECTION", flush=True)


if __name__ == "__main__":
    main()
