"""Worker process for tests/test_multiprocess.py (gloo, CPU only).

Environment: RANK, WORLD_SIZE, MASTER_ADDR, MASTER_PORT, MODE, OUT (a
directory for this rank's JSON result), N_STREAMS.
"""

import importlib
import json
import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    mode, out = os.environ["MODE"], Path(os.environ["OUT"])
    n = int(os.environ.get("N_STREAMS", "10"))
    dp = importlib.import_module("go-whistle_b200.dp")
    import torch.distributed as dist

    if mode == "max":
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
        v = dp.max_over_ranks(float(10 * rank + 1))
        dist.barrier()
        dist.destroy_process_group()
        (out / f"{rank}.json").write_text(json.dumps({"max": v}))
        return
    store = dist.TCPStore(os.environ["MASTER_ADDR"], int(os.environ["MASTER_PORT"]), world, rank == 0,
                          timeout=timedelta(seconds=30))
    mine = dp.shard(n, world, rank)
    if mode == "crash" and rank == world - 1:
        raise SystemExit(3)  # this rank dies before publishing its shard
    results = {s: 1000 + s for s in mine}
    g = dp.gather_results(store, world, rank, n, results, timeout_s=3.0)
    if rank == 0:
        (out / "0.json").write_text(json.dumps({"results": {str(k): v for k, v in g.results.items()},
                                                 "missing_ranks": g.missing_ranks,
                                                 "missing_streams": g.missing_streams}))


if __name__ == "__main__":
    main()
