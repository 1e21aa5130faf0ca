"""Multi-rank host logic on the CPU: cost-balanced sequence / request
assignment, shard rebasing and the variable-size output gather, run as two
gloo ranks.  Each rank computes its share with the numpy oracle (the
per-sequence math is independent, so the gathered result must equal the
single-process oracle); the GPU kernels themselves are covered by the
gpu-marked parity tests."""
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import sharding as S
from oracle import attention_oracle as O

LENS = [17, 128, 300, 511, 0, 5, 64, 1, 200]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_lpt_assign_balances_and_is_deterministic():
    costs = [10, 9, 8, 7, 6, 5, 4, 3, 2, 1]
    owner = S.lpt_assign(costs, 3)
    loads = [sum(c for c, o in zip(costs, owner) if o == r) for r in range(3)]
    assert max(loads) - min(loads) <= max(costs) and sorted(loads) == [18, 18, 19]
    assert owner == S.lpt_assign(costs, 3)
    assert S.lpt_assign([], 4) == []
    assert S.lpt_assign([5, 5], 1) == [0, 0]


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_varlen_shards_partition_the_batch(world):
    cu = [0] + np.cumsum(LENS).tolist()
    seen_seqs, seen_rows = [], []
    for r in range(world):
        sh = S.shard_varlen(cu, world, r)
        assert sh.seq_ids == sorted(sh.seq_ids)
        assert int(sh.cu_seqlens[-1]) == sh.token_index.numel()
        for j, s in enumerate(sh.seq_ids):
            rows = sh.token_index[int(sh.cu_seqlens[j]):int(sh.cu_seqlens[j + 1])].tolist()
            assert rows == list(range(cu[s], cu[s + 1]))
        seen_seqs += sh.seq_ids
        seen_rows += sh.token_index.tolist()
    assert sorted(seen_seqs) == list(range(len(LENS)))
    assert sorted(seen_rows) == list(range(cu[-1]))


def test_request_shards_partition_the_batch():
    ctx = [1, 8192, 77, 4096, 0, 3000, 129, 64]
    got = sorted(sum((S.shard_requests(ctx, 3, r).tolist() for r in range(3)), []))
    assert got == list(range(len(ctx)))


def _init(rank, world, port):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))


def _prefill_worker(rank, world, port, q_path):
    _init(rank, world, port)
    try:
        g = torch.Generator().manual_seed(5)
        T, H, Hkv, D = sum(LENS), 4, 2, 16
        q = torch.randn(T, H, D, generator=g, dtype=torch.float64)
        k = torch.randn(T, Hkv, D, generator=g, dtype=torch.float64)
        v = torch.randn(T, Hkv, D, generator=g, dtype=torch.float64)
        cu = [0] + np.cumsum(LENS).tolist()
        sh = S.shard_varlen(cu, world, rank)
        out, lse = O.prefill(sh.take(q).numpy(), sh.take(k).numpy(), sh.take(v).numpy(), sh.cu_seqlens.numpy())
        full_out = S.gather_rows(torch.from_numpy(out), sh.token_index, T)
        full_lse = S.gather_rows(torch.from_numpy(lse), sh.token_index, T, dst=0)
        assert (full_lse is None) == (rank != 0)
        if rank == 0:
            torch.save({"out": full_out, "lse": full_lse}, q_path)
    finally:
        dist.destroy_process_group()


def _decode_worker(rank, world, port, q_path):
    _init(rank, world, port)
    try:
        g = torch.Generator().manual_seed(9)
        B, H, Hkv, D, P, pool = 6, 4, 2, 16, 16, 100
        ctx = torch.tensor([1, 100, 33, 0, 16, 250], dtype=torch.int32)
        bt = torch.randperm(pool, generator=g)[: B * 16].reshape(B, 16).to(torch.int32)
        q = torch.randn(B, H, D, generator=g, dtype=torch.float64)
        kc = torch.randn(pool, Hkv, P, D, generator=g, dtype=torch.float64)
        vc = torch.randn(pool, Hkv, P, D, generator=g, dtype=torch.float64)
        ids = S.shard_requests(ctx, world, rank)
        out, _ = O.paged_decode(q[ids].numpy(), kc.numpy(), vc.numpy(), bt[ids].numpy(), ctx[ids].numpy(), P)
        full = S.gather_rows(torch.from_numpy(out), ids, B)
        if rank == 0:
            torch.save({"out": full}, q_path)
    finally:
        dist.destroy_process_group()


def _gather_forms_worker(rank, world, port, q_path):
    _init(rank, world, port)
    try:
        rows = [3, 5][rank]
        row0 = [0, 3][rank]
        local = torch.arange(row0, row0 + rows, dtype=torch.float32)[:, None] * torch.ones(1, 4)
        a = S.gather_rows(local, row0, 8)                                    # contiguous offsets
        b = S.gather_rows(local, torch.arange(row0, row0 + rows), 8, dst=1)  # index tensors, to rank 1
        c = S.gather_rows(local, row0 if rank == 0 else torch.arange(row0, row0 + rows), 8)  # mixed
        if rank == 1:
            torch.save({"a": a, "b": b, "c": c}, q_path)
        else:
            assert b is None
    finally:
        dist.destroy_process_group()


def test_two_rank_gather_forms(tmp_path):
    res = _run(_gather_forms_worker, 2, tmp_path)
    want = torch.arange(8, dtype=torch.float32)[:, None] * torch.ones(1, 4)
    for key in "abc":
        assert torch.equal(res[key], want), key


def _concat_worker(rank, world, port, q_path):
    _init(rank, world, port)
    try:
        rows = [5, 2, 0][rank]  # uneven blocks, one empty
        start = [0, 5, 7][rank]
        local = torch.arange(start, start + rows, dtype=torch.float32)[:, None] * torch.ones(1, 3)
        a = S.concat_rows(local)
        b = S.concat_rows(local, dst=2)
        if rank == 2:
            torch.save({"a": a, "b": b}, q_path)
        else:
            assert b is None
    finally:
        dist.destroy_process_group()


def test_three_rank_concat_uneven_blocks(tmp_path):
    res = _run(_concat_worker, 3, tmp_path)
    want = torch.arange(7, dtype=torch.float32)[:, None] * torch.ones(1, 3)
    assert torch.equal(res["a"], want) and torch.equal(res["b"], want)


def _planned_worker(rank, world, port, q_path):
    _init(rank, world, port)
    try:
        # the decode sharding plan, computed identically on every rank
        ctx = [1, 8192, 77, 4096, 0, 3000, 129, 64, 5000, 2]
        ids = [S.shard_requests(ctx, world, r) for r in range(world)]
        gather = S.PlannedGather([len(i) for i in ids], ids)
        local = ids[rank].to(torch.float32)[:, None] * torch.ones(1, 3) + 0.5
        a = gather(local)
        b = gather(local * 2)        # buffers reused
        c = S.PlannedGather([2, 0, 3][:world])(torch.full(([2, 0, 3][rank], 2), float(rank)))  # rank order
        d = S.PlannedGather([len(i) for i in ids], ids, dst=0)(local)  # to rank 0 only
        assert (d is None) == (rank != 0)
        if rank == 0:
            torch.save({"a": a, "b": b, "c": c, "d": d}, q_path)
    finally:
        dist.destroy_process_group()


def test_three_rank_planned_gather(tmp_path):
    """One collective, sizes from the sharding plan: rows land in global
    request order; without row numbers, blocks are concatenated by rank."""
    res = _run(_planned_worker, 3, tmp_path)
    want = torch.arange(10, dtype=torch.float32)[:, None] * torch.ones(1, 3) + 0.5
    assert torch.equal(res["a"], want)
    assert torch.equal(res["b"], want * 2)
    assert torch.equal(res["d"], want)
    assert torch.equal(res["c"], torch.tensor([[0.0, 0.0], [0.0, 0.0], [2.0, 2.0], [2.0, 2.0], [2.0, 2.0]]))


def _run(worker, world, tmp_path):
    path = str(tmp_path / "result.pt")
    mp.spawn(worker, args=(world, _free_port(), path), nprocs=world, join=True)
    return torch.load(path)


def test_two_rank_prefill_gather_matches_single_process(tmp_path):
    res = _run(_prefill_worker, 2, tmp_path)
    g = torch.Generator().manual_seed(5)
    T, H, Hkv, D = sum(LENS), 4, 2, 16
    q = torch.randn(T, H, D, generator=g, dtype=torch.float64)
    k = torch.randn(T, Hkv, D, generator=g, dtype=torch.float64)
    v = torch.randn(T, Hkv, D, generator=g, dtype=torch.float64)
    out, lse = O.prefill(q.numpy(), k.numpy(), v.numpy(), [0] + np.cumsum(LENS).tolist())
    # same per-sequence float64 math; BLAS may block differently for the
    # shard's array layout, hence a 1e-12 relative bound rather than bit equality
    np.testing.assert_allclose(res["out"].numpy(), out, rtol=1e-12, atol=1e-13)
    np.testing.assert_allclose(res["lse"].numpy(), lse, rtol=1e-12, atol=1e-13)


def test_two_rank_decode_gather_matches_single_process(tmp_path):
    res = _run(_decode_worker, 2, tmp_path)
    g = torch.Generator().manual_seed(9)
    B, H, Hkv, D, P, pool = 6, 4, 2, 16, 16, 100
    ctx = torch.tensor([1, 100, 33, 0, 16, 250], dtype=torch.int32)
    bt = torch.randperm(pool, generator=g)[: B * 16].reshape(B, 16).to(torch.int32)
    q = torch.randn(B, H, D, generator=g, dtype=torch.float64)
    kc = torch.randn(pool, Hkv, P, D, generator=g, dtype=torch.float64)
    vc = torch.randn(pool, Hkv, P, D, generator=g, dtype=torch.float64)
    out, _ = O.paged_decode(q.numpy(), kc.numpy(), vc.numpy(), bt.numpy(), ctx.numpy(), P)
    np.testing.assert_allclose(res["out"].numpy(), out, rtol=1e-12, atol=1e-13)
