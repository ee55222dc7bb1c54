"""Multi-GPU host logic (replicas, no data-path collective) on CPU gloo ranks.

The engine runs one replica per GPU; the only cross-rank steps are a barrier,
the max over ranks of the timed region, and rank 0 creating the model file
the other ranks read.  These tests run that code with the gloo backend and
world size 2 (and a rank that dies, to check the others end with an error
rather than wait forever).
"""
import os
import socket
import sys
import time

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "rf-detr.cpp_b200"))

from rfdetr_b200 import replicas  # noqa: E402


def test_shard_covers_every_item_once():
    for n in (0, 1, 7, 32, 256, 1000):
        for world in range(1, 9):
            seen = []
            sizes = []
            for r in range(world):
                lo, hi = replicas.shard(n, r, world)
                assert 0 <= lo <= hi <= n
                seen.extend(range(lo, hi))
                sizes.append(hi - lo)
            assert seen == list(range(n))
            assert max(sizes) - min(sizes) <= 1


def test_shard_rejects_bad_arguments():
    for args in ((4, 2, 2), (4, -1, 2), (4, 0, 0), (-1, 0, 1)):
        with pytest.raises(ValueError):
            replicas.shard(*args)


def test_rank_info_from_env():
    assert replicas.RankInfo.from_env({}) == replicas.RankInfo(0, 1, 0)
    assert replicas.RankInfo.from_env({"RANK": "3", "WORLD_SIZE": "4", "LOCAL_RANK": "1"}) == \
        replicas.RankInfo(3, 4, 1)
    with pytest.raises(ValueError):
        replicas.RankInfo.from_env({"RANK": "4", "WORLD_SIZE": "4"})


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, tmpdir, mode, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, os.path.join(ROOT, "rf-detr.cpp_b200"))
    from rfdetr_b200 import replicas as R
    info = R.RankInfo.from_env()
    res = {"rank": rank}
    try:
        with R.ProcessGroup(info, "gloo", timeout_s=5.0 if mode == "die" else 60.0) as pg:
            if mode == "die" and rank == 1:
                os._exit(3)  # leaves between steps, without joining the barrier
            path = os.path.join(tmpdir, "model.bin")

            def make(tmp):
                time.sleep(0.5)  # the other rank must wait for the finished file
                with open(tmp, "w") as f:
                    f.write("made by rank 0")
            R.create_once(path, make, pg)
            with open(path) as f:
                res["file"] = f.read()
            res["max"] = pg.max_over_ranks(10.0 * rank + 1.0)
            res["gathered"] = pg.gather_to_rank0(float(rank))
            res["shard"] = R.shard(256, info.rank, info.world)
            pg.barrier()
    except Exception as e:  # noqa: BLE001 - reported to the parent
        res["error"] = type(e).__name__
    out.put(res)


def _run(world, mode, tmp_path, timeout=90):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, str(tmp_path), mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    deadline = time.time() + timeout
    expected = world - (1 if mode == "die" else 0)
    while len(results) < expected and time.time() < deadline:
        try:
            results.append(q.get(timeout=1.0))
        except Exception:  # noqa: BLE001 - queue.Empty
            pass
    for p in procs:
        p.join(timeout=max(1.0, deadline - time.time()))
        if p.is_alive():
            p.kill()
    return sorted(results, key=lambda r: r["rank"]), [p.exitcode for p in procs]


def test_two_gloo_ranks(tmp_path):
    res, codes = _run(2, "ok", tmp_path)
    assert codes == [0, 0], codes
    assert [r.get("error") for r in res] == [None, None], res
    assert all(r["file"] == "made by rank 0" for r in res)
    assert all(r["max"] == 11.0 for r in res)
    assert res[0]["gathered"] == [0.0, 1.0] and res[1]["gathered"] is None
    assert res[0]["shard"] == (0, 128) and res[1]["shard"] == (128, 256)


def test_dead_rank_ends_the_others_with_an_error(tmp_path):
    t0 = time.time()
    res, codes = _run(2, "die", tmp_path, timeout=120)
    assert codes[1] == 3
    assert len(res) == 1 and res[0]["rank"] == 0
    assert res[0].get("error"), res
    assert time.time() - t0 < 110
