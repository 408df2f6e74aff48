"""Multi-GPU host logic on CPU: sequence sharding and the KV-range split with
the (m, l, o) exchange, run as two gloo ranks.  The partial states come from
the CPU oracle, so this checks the partition + exchange + merge, not a kernel."""
import os
import socket

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


@pytest.mark.timeout(120)
def test_kv_range_split_merge_two_gloo_ranks():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, 7, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=100)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    errs = dict(q.get(timeout=5) for _ in range(2))
    assert max(errs.values()) < 1e-5, errs


def _dropout_main(rank, world, port, q):
    """Rank 1 leaves between steps; rank 0 learns of it from the store before
    its next collective instead of hanging in it."""
    import datetime
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    store = dist.distributed_c10d._get_default_store()
    x = torch.ones(4)
    dist.all_reduce(x)  # step 1 with both ranks
    if rank == 1:
        store.set("rank1_leaving", "1")
        q.put((rank, "left"))
        q.close()
        q.join_thread()
        os._exit(0)
    # rank 0: check the store (heartbeat) before the next step's collective
    store.wait(["rank1_leaving"], datetime.timedelta(seconds=20))
    q.put((rank, "saw-departure" if store.get("rank1_leaving") == b"1" else "missed"))
    q.close()
    q.join_thread()
    os._exit(0)


@pytest.mark.timeout(120)
def test_rank_departure_detected_on_host():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dropout_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=100)
    for p in procs:
        if p.is_alive():
            p.kill()
    res = dict(q.get(timeout=5) for _ in range(2))
    assert res == {0: "saw-departure", 1: "left"}
