"""Host-side multi-rank logic on CPU: world-size-2 gloo ranks shard the
(batch, head) pairs, regenerate their shards from the seed, compute them (the
oracle stands in for the kernel here -- the CUDA path is tested on the GPU),
gather on rank 0 and all-reduce the verification statistics.  The gathered
result must equal the single-process result exactly."""

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cs348k_fast_attention_grammar_b200.inputs import make_qkv, pair_seed, pair_tensor
from cs348k_fast_attention_grammar_b200.parallel import (owner_of, reduce_error_stats,
                                                         shard_range, verify_pairs)

CFG = dict(B=2, H=4, S=96, D=64, causal=True, seed=9, amp=0.5)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _compute(q, k, v, causal):
    import oracle
    out = np.empty(q.shape, dtype=np.float64)
    for i in range(q.shape[1]):
        out[0, i] = oracle.attention_pair(q[0, i].float().numpy(), k[0, i].float().numpy(),
                                          v[0, i].float().numpy(), causal=causal)
    return torch.from_numpy(out)


def _worker(rank, world, port, result_path, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=30))
    try:
        npairs = CFG["B"] * CFG["H"]
        pairs = shard_range(npairs, world, rank)
        q, k, v = make_qkv(CFG, pairs, "cpu")
        o = _compute(q, k, v, CFG["causal"])
        if rank == fail_rank:
            raise RuntimeError("injected rank failure")
        bufs = [torch.empty_like(o) for _ in range(world)] if rank == 0 else None
        dist.gather(o, gather_list=bufs, dst=0)
        mx, sm, cnt = 0.0, 0.0, 0
        for p in verify_pairs(npairs, 3):
            if p in pairs:
                i = p - pairs.start
                d = (o[0, i] - _compute(q[:, i:i + 1], k[:, i:i + 1], v[:, i:i + 1],
                                        CFG["causal"])[0, 0]).abs()
                mx, sm, cnt = max(mx, d.max().item()), sm + d.sum().item(), cnt + d.numel()
        stats = reduce_error_stats(mx, sm, cnt, "cpu")
        if rank == 0:
            torch.save({"o": torch.cat(bufs, dim=1), "stats": stats}, result_path)
    finally:
        dist.destroy_process_group()


def test_shard_ranges_cover_exactly():
    for n, w in [(128, 1), (128, 2), (128, 8), (2048, 8), (10, 3)]:
        seen = [p for r in range(w) for p in shard_range(n, w, r)]
        assert seen == list(range(n))
        assert all(owner_of(p, n, w) == r for r in range(w) for p in shard_range(n, w, r))


def test_pair_generation_is_independent_of_sharding():
    a = make_qkv(CFG, range(8), "cpu")[1]
    b = make_qkv(CFG, range(4, 8), "cpu")[1]
    assert torch.equal(a[:, 4:], b)
    assert pair_seed(1, "q", 5) != pair_seed(1, "k", 5) != pair_seed(2, "q", 5)
    t = pair_tensor(2, "q", 3, 64, 32, 0.5, "cpu")
    assert t.dtype == torch.bfloat16 and abs(t.float().std().item() - 0.5) < 0.05


def test_two_gloo_ranks_match_single_process(tmp_path):
    path = str(tmp_path / "res.pt")
    mp.start_processes(_worker, args=(2, _free_port(), path, -1), nprocs=2, join=True,
                       start_method="spawn")
    res = torch.load(path)
    q, k, v = make_qkv(CFG, range(CFG["B"] * CFG["H"]), "cpu")
    single = _compute(q, k, v, CFG["causal"])
    assert torch.equal(res["o"], single)
    assert res["stats"]["max_abs"] == 0.0 and res["stats"]["elements"] == 3 * 96 * 64


def test_rank_failure_surfaces_as_error(tmp_path):
    """A rank that raises between steps ends the job with an error on the
    host (no hang): the surviving rank's gather fails or the launcher reports
    the failed process."""
    path = str(tmp_path / "res.pt")
    with pytest.raises(Exception):
        mp.start_processes(_worker, args=(2, _free_port(), path, 1), nprocs=2, join=True,
                           start_method="spawn")
    assert not os.path.exists(path)


MLP_CFG = dict(M=96, K=64, N=128, seed=13)


def _mlp_worker(rank, world, port, result_path):
    """The MLP line's multi-rank logic (bench.py --config cfg3 under torchrun):
    rows of X sharded over the ranks with replicated weights, every rank
    regenerating the same seeded tensors, Y gathered on rank 0 and a seeded
    spot check of rows reduced over the ranks (the oracle stands in for the
    GEMM kernels here)."""
    import oracle
    from cs348k_fast_attention_grammar_b200.inputs import make_mlp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=30))
    try:
        x_full, w1, w2 = make_mlp(MLP_CFG, "cpu")
        rows = shard_range(MLP_CFG["M"], world, rank)
        x = x_full[rows.start:rows.stop]
        y = torch.from_numpy(oracle.mlp(x.float().numpy(), w1.float().numpy(),
                                        w2.float().numpy(), act="gelu_tanh"))
        bufs = [torch.empty_like(y) for _ in range(world)] if rank == 0 else None
        dist.gather(y.contiguous(), gather_list=bufs, dst=0)
        sel = np.random.default_rng(rank).choice(len(rows), 8, replace=False)
        ref = oracle.mlp(x.float().numpy()[sel], w1.float().numpy(), w2.float().numpy(),
                         act="gelu_tanh")
        d = np.abs(y.numpy()[sel] - ref)
        stats = reduce_error_stats(float(d.max()), float(d.sum()), d.size, "cpu")
        if rank == 0:
            torch.save({"y": torch.cat(bufs, dim=0), "stats": stats}, result_path)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_mlp_row_split_matches_single_process(tmp_path):
    import oracle
    from cs348k_fast_attention_grammar_b200.inputs import make_mlp
    path = str(tmp_path / "mlp.pt")
    mp.start_processes(_mlp_worker, args=(2, _free_port(), path), nprocs=2, join=True,
                       start_method="spawn")
    res = torch.load(path)
    x, w1, w2 = make_mlp(MLP_CFG, "cpu")
    single = oracle.mlp(x.float().numpy(), w1.float().numpy(), w2.float().numpy(),
                        act="gelu_tanh")
    assert res["y"].shape == (MLP_CFG["M"], MLP_CFG["K"])
    np.testing.assert_array_equal(res["y"].numpy(), single)
    assert res["stats"]["max_abs"] == 0.0 and res["stats"]["elements"] == 2 * 8 * MLP_CFG["K"]


def _spread_worker(rank, world, port, result_path):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=30))
    try:
        got = bench.rank_ms_spread(1.0 + rank, world, "cpu")
        torch.save(got, f"{result_path}.{rank}")
    finally:
        dist.destroy_process_group()


def test_bench_rank_spread_on_two_gloo_ranks(tmp_path):
    """bench.py's step time is the slowest rank's; the line also reports the
    fastest.  Every rank gets both from one all-reduce."""
    out = str(tmp_path / "spread")
    mp.spawn(_spread_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    for r in range(2):
        assert torch.load(f"{out}.{r}") == (2.0, 1.0)
