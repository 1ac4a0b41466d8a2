"""Multi-rank layer on CPU with the gloo backend (world size 2): shard ranges,
the to-root gather of BBOs and int64 positions against a single run over all
markets, and a rank that dies before the gather."""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from astra_cuda.sharding import shard_range

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_shard_range_covers_exactly():
    for total in (0, 1, 7, 1000, 1_000_003):
        for world in (1, 2, 3, 4, 8):
            got = [shard_range(r, world, total) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == total
            for (a, b), (c, d) in zip(got, got[1:]):
                assert b == c and b >= a
            sizes = [b - a for a, b in got]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(2, 2, 10)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, total, steps, mode, q):
    for p in (os.path.join(ROOT, "astra-cuda_b200"), os.path.join(ROOT, "oracle")):
        sys.path.insert(0, p)
    from datetime import timedelta
    import torch.distributed as dist
    import oracle
    from astra_cuda import workloads
    from astra_cuda.sharding import gather_to_root, shard_range
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=timedelta(seconds=8))
        c = workloads.CONFIGS[4]
        a, b = shard_range(rank, world, total)
        n = b - a
        mkt = oracle.OracleMarket(n, c["L"], 64, 32, c["C"])
        fills, bbos = mkt.new_fill_batch(), mkt.new_bbo_batch()
        gen = oracle.OracleQuoteGen(c["gen"], a, n)
        pos = np.zeros((n, c["C"], 2), np.int64)
        for _ in range(steps):
            mkt.add_two_sided_quotes(*gen.step(), fills, pos64=pos)
        mkt.get_bbos(bbos)
        bbo = torch.from_numpy(np.stack([bbos[k] for k in ("best_bid_prices", "best_bid_sizes",
                                                            "best_ask_prices", "best_ask_sizes")]))
        if mode == "die" and rank == 1:
            q.put((rank, "left"))
            q.close()
            q.join_thread()  # flush the message before leaving
            os._exit(0)  # leaves between steps, before the collective
        try:
            out = gather_to_root([(bbo, 1), torch.from_numpy(pos)])
        except Exception as ex:  # the survivor must see an error, not hang
            q.put((rank, "error:" + type(ex).__name__))
            return
        if rank == 0:
            q.put((rank, (out[0].numpy(), out[1].numpy())))
        else:
            q.put((rank, None))
        dist.destroy_process_group()
    except Exception as ex:
        q.put((rank, "exc:" + repr(ex)))


def _run(mode, total=300, steps=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, total, steps, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, v = q.get(timeout=120)
        res[r] = v
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


def test_gloo_gather_equals_single_run():
    import oracle
    from astra_cuda import workloads
    total, steps = 300, 60
    res = _run("ok", total, steps)
    assert not isinstance(res[0], str), res
    bbo, pos = res[0]
    c = workloads.CONFIGS[4]
    mkt = oracle.OracleMarket(total, c["L"], 64, 32, c["C"])
    fills, bbos = mkt.new_fill_batch(), mkt.new_bbo_batch()
    gen = oracle.OracleQuoteGen(c["gen"], 0, total)
    p1 = np.zeros((total, c["C"], 2), np.int64)
    for _ in range(steps):
        mkt.add_two_sided_quotes(*gen.step(), fills, pos64=p1)
    mkt.get_bbos(bbos)
    want = np.stack([bbos[k] for k in ("best_bid_prices", "best_bid_sizes", "best_ask_prices",
                                       "best_ask_sizes")])
    np.testing.assert_array_equal(bbo, want)
    np.testing.assert_array_equal(pos, p1)


def test_gloo_gather_rank_leaves():
    """Rank 1 leaves between steps; rank 0's gather ends with an error from
    the process-group timeout instead of waiting forever."""
    res = _run("die")
    assert res[1] == "left"
    assert isinstance(res[0], str) and res[0].startswith("error:"), res
