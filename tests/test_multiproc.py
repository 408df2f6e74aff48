"""Multi-GPU host logic on CPU: sequence sharding and the KV-range split with
the (m, l, o) exchange, run as two gloo ranks.  The partial states come from
the CPU oracle, so this checks the partition + exchange + merge, not a kernel."""
import os
import socket
import time

import numpy as np
import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_lpt_shard_balances_and_covers():
    from qwanto_b200.sharding import balanced_count_shard, lpt_shard
    rng = np.random.default_rng(0)
    lens = rng.integers(1024, 8193, size=256)
    for ranks in (1, 2, 4, 8):
        parts = lpt_shard(lens, ranks)
        assert sorted(i for p in parts for i in p) == list(range(256))
        loads = [int(lens[p].sum()) for p in parts]
        assert max(loads) - min(loads) <= int(lens.max())
        eq = balanced_count_shard(lens, ranks)
        assert all(len(p) == 256 // ranks for p in eq)
        assert sorted(i for p in eq for i in p) == list(range(256))
        loads = [int(lens[p].sum()) for p in eq]
        assert (max(loads) - min(loads)) / np.mean(loads) < 0.05


def test_kv_ranges_page_aligned():
    from qwanto_b200.sharding import kv_ranges
    for total, ranks, P in [(131072, 8, 64), (1000, 3, 16), (64, 4, 64)]:
        r = kv_ranges(total, ranks, P)
        assert r[0][0] == 0 and r[-1][1] == total
        for (a, b), (c, d) in zip(r, r[1:]):
            assert b == c and a % P == 0
        assert all(b >= a for a, b in r)


def _rank_main(rank, world, port, seed, q):
    import torch
    import torch.distributed as dist
    from oracle import oracle as O
    from qwanto_b200.sharding import gather_and_merge, kv_ranges
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        H, HK, T, P = 12, 2, 700, 64
        pool = O.Pool(2, 1, HK, P, 32, 1, 32)
        assert pool.append([0], [T]) == 0
        for t in range(T):
            pool.write(0, 0, t, O.gen_row(seed, 2, 0, 0, t, HK * 128), O.gen_row(seed, 3, 0, 0, t, HK * 128))
        qv = O.gen_row(seed, 1, 0, 0, T - 1, H * 128)
        t0, t1 = kv_ranges(T, world, P)[rank]
        m = np.zeros(H, np.float32)
        l = np.zeros(H, np.float32)
        o = np.zeros((H, 128), np.float32)
        O.lib().qor_partial_attention(__import__("ctypes").byref(pool.p), 0, 0, t0, t1, O._ptr(qv, O.f32p), H,
                                      1.0 / np.sqrt(128.0), O._ptr(m, O.f32p), O._ptr(l, O.f32p), O._ptr(o, O.f32p))
        out = torch.zeros((H, 128))
        gather_and_merge(torch.from_numpy(m), torch.from_numpy(l), torch.from_numpy(o), out, H)
        full = pool.attention(0, 0, T, qv, H, 1.0 / np.sqrt(128.0))
        q.put((rank, float(np.abs(out.numpy() - full).max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(180)
@pytest.mark.parametrize("world", [2, 4])
def test_kv_range_split_merge_gloo_ranks(world):
    """One context split into `world` page-aligned ranges, a partial (m, l, o)
    per rank, all-gathered and merged on every rank: equal to the whole
    attention on every rank (the host side of the split-KV path)."""
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, 7, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=150)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0] * world, codes
    errs = dict(q.get(timeout=5) for _ in range(world))
    assert max(errs.values()) < 1e-5, errs


def _silent_exit_main(rank, world, port, q):
    """Rank 1 runs one step and then exits between steps without a word (no
    store key, no message).  Rank 0 finds it through the heartbeat before its
    next collective, then confirms that a short process-group timeout ends a
    collective with the lost rank in an error instead of a hang."""
    import datetime
    import torch
    import torch.distributed as dist
    from qwanto_b200.health import Heartbeat, RankLostError
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    store = dist.distributed_c10d._get_default_store()
    hb = Heartbeat(store, rank, world, interval=0.02).start()
    x = torch.ones(4)
    hb.check_peers(timeout=5.0)
    dist.all_reduce(x)  # step 1 with both ranks
    if rank == 1:
        os._exit(0)  # silent: the heartbeat thread dies with the process
    time.sleep(0.3)
    try:
        hb.check_peers(timeout=1.0)
        verdict = "missed"
    except RankLostError as e:
        verdict = f"lost {e.ranks}"
    t0 = time.monotonic()
    try:
        dist.all_reduce(x)  # what a rank without the check would do
        coll = "completed"
    except Exception:
        coll = "error"
    q.put((rank, verdict, coll, time.monotonic() - t0))
    q.close()
    q.join_thread()
    os._exit(0)


@pytest.mark.timeout(120)
def test_silent_rank_exit_detected_by_heartbeat():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_silent_exit_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=100)
    for p in procs:
        if p.is_alive():
            p.kill()
    rank, verdict, coll, waited = q.get(timeout=5)
    assert (rank, verdict) == (0, "lost [1]")
    assert coll == "error" and waited < 30


def test_heartbeat_sees_live_peers_and_stale_ones():
    """The check itself on one process: a peer key that keeps moving passes,
    one that stands still raises after the timeout, a missing one too."""
    import threading
    from torch.distributed import HashStore
    from qwanto_b200.health import Heartbeat, RankLostError
    store = HashStore()
    a = Heartbeat(store, 0, 3, interval=0.01).start()
    b = Heartbeat(store, 1, 3, interval=0.01).start()
    try:
        with pytest.raises(RankLostError) as ei:
            a.check_peers(timeout=0.2)  # rank 2 never started
        assert ei.value.ranks == [2]
        store.set("qwn_hb/2", "5")  # present but frozen
        with pytest.raises(RankLostError) as ei:
            a.check_peers(timeout=0.2)
        assert ei.value.ranks == [2]
        stop = threading.Event()

        def beat():
            n = 6
            while not stop.is_set():
                store.set("qwn_hb/2", str(n))
                n += 1
                time.sleep(0.01)
        t = threading.Thread(target=beat)
        t.start()
        try:
            a.check_peers(timeout=2.0)
            b.check_peers(timeout=2.0)
        finally:
            stop.set()
            t.join()
    finally:
        a.stop()
        b.stop()
