"""Split-KV decode with the exchange fused into the attention kernel
(qwn_kv_decode_split): one rank against the full decode and the oracle, a
rank whose peers never arrive (bounded wait, status bit, pool still usable),
and two ranks on two GPUs (skipped on a one-GPU box)."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from kvharness import Twin, assert_close

pytestmark = pytest.mark.gpu

H, HK, P = 48, 8, 64


def _query(torch, qb, seed, pos):
    q = torch.empty((1, H * 128), dtype=torch.float32, device="cuda")
    p = torch.tensor([pos], dtype=torch.int32, device="cuda")
    qb.generate_rows(q, 1, H * 128, 1, seed, 0, None, p)
    return q


@pytest.mark.parametrize("codec", [2, 4, 5])
def test_split_one_rank_matches_decode_and_oracle(cuda, codec):
    import qwanto_b200 as qb
    from qwanto_b200._lib import ST_PEER_TIMEOUT
    from qwanto_b200.exchange import PeerExchange
    torch = cuda
    tw = Twin(cuda, codec, layers=1, kv_heads=HK, page_tokens=P, total_pages=80, max_seqs=1, max_pages=80,
              query_heads=H, perm_seed=4, seed=23)
    ex = PeerExchange(H, device=0, timeout_ns=1_000_000_000)
    try:
        tw.prefill([0], [3000])
        q = _query(torch, qb, 23, 2999)
        full = torch.zeros_like(q)
        tw.gpu.decode(0, 1, H, q, full)
        out = torch.full_like(q, float("nan"))
        tw.gpu.decode_split(0, H, q, out, ex)
        torch.cuda.synchronize()
        assert (tw.gpu.check() & ST_PEER_TIMEOUT) == 0
        assert_close(out.cpu().numpy(), full.cpu().numpy(), f"codec {codec} split x1 vs decode")
        ref = tw.ora.attention(0, 0, 3000, tw.row(1, 0, 0, 2999, H * 128), H, 1.0 / np.sqrt(128.0))
        assert_close(out.cpu().numpy().reshape(H, 128), ref, f"codec {codec} split x1 vs oracle")
        # a sub-range equals the partial of that range, merged alone
        m = torch.zeros((1, H), device="cuda")
        l = torch.zeros((1, H), device="cuda")
        o = torch.zeros((1, H, 128), device="cuda")
        tw.gpu.partial(0, 1, H, q, m[0], l[0], o[0], t_begin=704, t_end=2112)
        sub = torch.zeros((H, 128), device="cuda")
        qb.merge_partials(1, H, m, l, o, sub)
        out2 = torch.full_like(q, float("nan"))
        tw.gpu.decode_split(0, H, q, out2, ex, t_begin=704, t_end=2112)
        torch.cuda.synchronize()
        assert_close(out2.cpu().numpy().reshape(H, 128), sub.cpu().numpy(), f"codec {codec} split sub-range")
        # the newest token stored by the split call itself (range to the end)
        tw.gpu.seq_append(1)
        assert tw.ora.append([0], [1]) == 0
        W = HK * 128
        pos = torch.tensor([3000], dtype=torch.int32, device="cuda")
        k = torch.empty((1, W), dtype=torch.float32, device="cuda")
        v = torch.empty((1, W), dtype=torch.float32, device="cuda")
        qb.generate_rows(k, 1, W, 2, 23, 0, None, pos)
        qb.generate_rows(v, 1, W, 3, 23, 0, None, pos)
        q3 = _query(torch, qb, 23, 3000)
        out3 = torch.full_like(q3, float("nan"))
        tw.gpu.decode_split(0, H, q3, out3, ex, key=k, value=v)
        torch.cuda.synchronize()
        assert tw.gpu.check() == 0
        assert tw.ora.write(0, 0, 3000, tw.row(2, 0, 0, 3000, W), tw.row(3, 0, 0, 3000, W)) == 0
        ref3 = tw.ora.attention(0, 0, 3001, tw.row(1, 0, 0, 3000, H * 128), H, 1.0 / np.sqrt(128.0))
        assert_close(out3.cpu().numpy().reshape(H, 128), ref3, f"codec {codec} split x1 with append")
        tw.assert_state_equal()
        tw.assert_pages_equal()
    finally:
        torch.cuda.synchronize()
        ex.close()
        tw.close()


def test_split_peer_timeout_latches_and_pool_stays_usable(cuda):
    """Rank 0 of 2 whose peer never runs: every wait for the peer's flag runs
    into its 20 ms limit, the call latches PEER_TIMEOUT instead of hanging,
    and the next call on the same pool and context works."""
    import qwanto_b200 as qb
    from qwanto_b200._lib import ST_PEER_TIMEOUT
    from qwanto_b200.exchange import PeerExchange
    torch = cuda
    tw = Twin(cuda, 2, layers=1, kv_heads=HK, page_tokens=P, total_pages=40, max_seqs=1, max_pages=40,
              query_heads=H, seed=5)
    ex = PeerExchange.unreachable(H, device=0, world=2, timeout_ns=20_000_000)
    try:
        tw.prefill([0], [1500])
        q = _query(torch, qb, 5, 1499)
        out = torch.zeros_like(q)
        tw.gpu.decode_split(0, H, q, out, ex, t_begin=0, t_end=768)
        torch.cuda.synchronize()
        assert tw.gpu.check() & ST_PEER_TIMEOUT
        assert tw.gpu.check() == 0  # cleared by the read
        full = torch.zeros_like(q)
        tw.gpu.decode(0, 1, H, q, full)
        torch.cuda.synchronize()
        ref = tw.ora.attention(0, 0, 1500, tw.row(1, 0, 0, 1499, H * 128), H, 1.0 / np.sqrt(128.0))
        assert_close(full.cpu().numpy().reshape(H, 128), ref, "decode after a peer timeout")
        assert tw.gpu.check() == 0
    finally:
        torch.cuda.synchronize()
        ex.close()
        tw.close()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_rank_worker(rank, world, port, codec, ctx, result_q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        import qwanto_b200 as qb
        from qwanto_b200.exchange import PeerExchange
        from qwanto_b200.sharding import kv_ranges
        dev = torch.device("cuda", rank)
        pool = qb.KvPool(codec, 1, HK, P, ctx // P + 8, 1, ctx // P + 8, max_query_heads=H, permutation_seed=7,
                         device=rank)
        pool.prefill_synthetic([0], [ctx], 41)
        ex = PeerExchange(H, device=rank, timeout_ns=2_000_000_000)
        q = torch.empty((1, H * 128), dtype=torch.float32, device=dev)
        qb.generate_rows(q, 1, H * 128, 1, 41, 0, None, torch.tensor([ctx - 1], dtype=torch.int32, device=dev))
        full = torch.zeros_like(q)
        pool.decode(0, 1, H, q, full)
        a, b = kv_ranges(ctx, world, P)[rank]
        outs = []
        for _ in range(3):  # both parities and a reuse of the first
            out = torch.full_like(q, float("nan"))
            pool.decode_split(0, H, q, out, ex, t_begin=a, t_end=b if rank < world - 1 else 0)
            outs.append(out)
        torch.cuda.synchronize()
        status = pool.check()
        gathered = [torch.zeros_like(q) for _ in range(world)]
        dist.all_gather(gathered, outs[-1])
        same = all(torch.equal(g, gathered[0]) for g in gathered)
        err = max(float(((o - full).abs() - (1e-4 + 1e-3 * full.abs())).max()) for o in outs)
        dist.barrier()
        ex.close()
        pool.close()
        result_q.put((rank, status, same, err))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,ctx", [(2, 20000), (2, 131072), (4, 131072), (8, 131072)])
def test_split_n_gpus(cuda, world, ctx):
    """world ranks on world GPUs, one long sequence split into page ranges
    (131,072 tokens is the cfg4 context): every rank ends with the same
    rows, within tolerance of the one-GPU decode; both exchange parities."""
    torch = cuda
    codec = 2
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx_ = mp.get_context("spawn")
    q = ctx_.Queue()
    port = _free_port()
    procs = [ctx_.Process(target=_two_rank_worker, args=(r, world, port, codec, ctx, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    res = sorted(q.get(timeout=5) for _ in range(world))
    for rank, status, same, err in res:
        assert status == 0, f"rank {rank} status {status:#x}"
        assert same, "ranks disagree"
        assert err <= 0.0, f"rank {rank}: split output outside tolerance of the full decode ({err})"
