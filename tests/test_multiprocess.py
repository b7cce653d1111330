"""Data parallelism across processes, on the CPU: world-size
2 gloo ranks and a TCP store, launched as child processes. No GPU: the path
has no data-path collective; these check the host logic (shard map,
max-over-ranks timing, result gathering) and failure detection (a rank that
dies is reported as a missing shard instead of hanging the others)."""

from __future__ import annotations

import importlib
import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def launch(mode: str, world: int, out: Path, n: int = 10):
    port = free_port()
    procs = []
    for rank in range(world):
        env = dict(os.environ, RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(port), MODE=mode, OUT=str(out), N_STREAMS=str(n), CUDA_VISIBLE_DEVICES="")
        procs.append(subprocess.Popen([sys.executable, str(HERE / "mp_worker.py")], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT))
    codes = []
    for p in procs:
        try:
            p.wait(timeout=120)
        except subprocess.TimeoutExpired:
            p.kill()
            p.wait()
        codes.append(p.returncode)
    return codes


def test_shard_covers_every_stream_once():
    dp = importlib.import_module("go-whistle_b200.dp")
    for n in (0, 1, 7, 1024):
        for world in (1, 2, 3, 8):
            seen = sorted(s for r in range(world) for s in dp.shard(n, world, r))
            assert seen == list(range(n))
            sizes = [len(dp.shard(n, world, r)) for r in range(world)]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        dp.shard(4, 2, 2)


def test_max_over_ranks_gloo(tmp_path):
    codes = launch("max", 2, tmp_path)
    assert codes == [0, 0]
    for r in range(2):
        assert json.loads((tmp_path / f"{r}.json").read_text())["max"] == 11.0


def test_gather_all_shards(tmp_path):
    codes = launch("ok", 2, tmp_path, n=9)
    assert codes == [0, 0]
    got = json.loads((tmp_path / "0.json").read_text())
    assert got["missing_ranks"] == [] and got["missing_streams"] == []
    assert {int(k): v for k, v in got["results"].items()} == {s: 1000 + s for s in range(9)}


def test_dead_rank_reported_as_missing_shard(tmp_path):
    """The last rank exits before publishing; rank 0 finishes within its
    timeout and names the missing rank and its streams."""
    codes = launch("crash", 2, tmp_path, n=9)
    assert codes[0] == 0 and codes[1] == 3
    got = json.loads((tmp_path / "0.json").read_text())
    assert got["missing_ranks"] == [1]
    assert got["missing_streams"] == [1, 3, 5, 7]
    assert {int(k) for k in got["results"]} == {0, 2, 4, 6, 8}
