"""The multi-GPU bench path's host logic on CPU: two gloo ranks launched by torchrun.

bench.py runs one process per GPU over independent streams, with no collective on the data
path: the only cross-rank steps are the barriers and the max-over-ranks reduction of every
timing. Here two ranks run under `python -m torch.distributed.run` (the driver's launcher) with
the gloo backend on 127.0.0.1, and check:
- max_over_ranks hands every rank the slowest rank's time;
- the ranks' stream blocks are disjoint and cover [0, world * B), and a stream's synthetic
  audio depends only on its global index, so stream g sees the same tokens at any GPU count;
- without a process group the helpers return the local values.
A static check of bench.py adds that every model it builds is placed on the rank's own GPU
(device=local_rank): a model left on GPU 0 fails on every other rank, because its kernels are
then launched on a stream of another device.
"""
import ast
import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent

WORKER = r'''
import json, os, sys
sys.path.insert(0, {root!r})
import torch.distributed as dist
import bench
from svl import config, synth

rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
dist.init_process_group("gloo")
B = 3
slowest = bench.max_over_ranks(dist, 10.0 + rank, "cpu")
streams = list(bench.rank_streams(rank, B))
audio = synth.audio_tokens(config.stt_toy(), 4, seed=1 + streams[0], streams=B)
got = [None] * world
dist.all_gather_object(got, {{"rank": rank, "slowest": slowest, "streams": streams,
                              "audio": audio.tolist()}})
dist.barrier()
dist.destroy_process_group()
if rank == 0:
    print("RESULT " + json.dumps(got), flush=True)
'''


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks(tmp_path):
    script = tmp_path / "worker.py"
    script.write_text(WORKER.format(root=str(ROOT)))
    env = dict(os.environ, OMP_NUM_THREADS="1")
    r = subprocess.run(
        [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
         "--master-addr=127.0.0.1", f"--master-port={_free_port()}", str(script)],
        capture_output=True, text=True, timeout=300, env=env, cwd=str(tmp_path))
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    line = next(l for l in r.stdout.splitlines() if l.startswith("RESULT "))
    ranks = json.loads(line[len("RESULT "):])
    world, B = 2, 3
    assert [g["rank"] for g in ranks] == [0, 1]
    # Every rank sees the slowest rank's time.
    assert all(g["slowest"] == 11.0 for g in ranks)
    # Disjoint contiguous blocks covering all streams.
    streams = [s for g in ranks for s in g["streams"]]
    assert streams == list(range(world * B))
    # Stream g's audio equals the one-stream draw from seed 1 + g.
    from svl import config, synth

    stt = config.stt_toy()
    for g in ranks:
        audio = np.asarray(g["audio"], np.uint32)
        for j, s in enumerate(g["streams"]):
            np.testing.assert_array_equal(audio[:, j], synth.audio_tokens(stt, 4, seed=1 + s))


def test_helpers_without_process_group():
    sys.path.insert(0, str(ROOT))
    import bench

    assert bench.max_over_ranks(None, 2.5, "cpu") == 2.5
    assert list(bench.rank_streams(0, 4)) == [0, 1, 2, 3]
    assert list(bench.rank_streams(3, 2)) == [6, 7]


def test_bench_places_every_model_on_the_rank_gpu():
    tree = ast.parse((ROOT / "bench.py").read_text())
    built = []
    for node in ast.walk(tree):
        if isinstance(node, ast.Call):
            f = node.func
            name = f.attr if isinstance(f, ast.Attribute) else getattr(f, "id", "")
            if name in ("LanguageModel", "FlowLm", "Mimi", "Quantizer"):
                kw = {k.arg: k.value for k in node.keywords}
                built.append(name)
                assert "device" in kw and isinstance(kw["device"], ast.Name) and kw["device"].id == "local_rank", \
                    f"bench.py line {node.lineno}: {name}(...) without device=local_rank"
    assert {"LanguageModel", "FlowLm", "Mimi", "Quantizer"} <= set(built)
