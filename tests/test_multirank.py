"""CPU: the request-sharded multi-rank path of bench.py with world_size 2 on
gloo - each rank owns its own requests, timing is the max over ranks - and
the reference arm's output contract."""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, str(ROOT))
    import bench

    class Args:
        pass

    w, r, local = bench.dist_setup(Args())
    assert (w, r, local) == (world, rank, rank)
    bench.barrier(w)
    # each rank reports a different elapsed time; every rank must see the maximum
    got = bench.max_over_ranks(10.0 + rank, w)
    contexts = bench.contexts_for(r)
    Path(out_dir, f"rank{rank}.json").write_text(json.dumps({"max": got, "contexts": contexts}))
    import torch.distributed as dist

    dist.destroy_process_group()


def test_two_ranks_shard_requests_and_take_the_max_time(tmp_path):
    port = _free_port()
    mp.start_processes(_rank_main, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    r0 = json.loads((tmp_path / "rank0.json").read_text())
    r1 = json.loads((tmp_path / "rank1.json").read_text())
    assert r0["max"] == r1["max"] == 11.0
    # request-sharded: ranks draw different request sets of the same distribution
    assert r0["contexts"] != r1["contexts"]
    for c in (r0["contexts"], r1["contexts"]):
        assert len(c) == 64 and min(c) >= 64 and max(c) <= 2048


def test_reference_arm_prints_the_contract_line():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                           "--warmup", "0"], capture_output=True, text=True, env=env, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    line = json.loads(proc.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "seq-steps/s" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0
    torch.testing.assert_close(line["e2e"]["value"], line["value"])
