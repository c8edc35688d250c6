"""Multi-GPU host logic on CPU: gloo ranks (world size 2) shard a generated
workload by contiguous id range, search their shard exactly, rebase ids,
exchange top-k through ShardExchange.gather (the all-gather bench.py runs over
NCCL) and merge with the oracle's shard merge; the result must equal the exact
filtered top-k over the whole base set.  A second test makes one rank leave
before the exchange and checks the other ends with an error instead of
waiting forever."""
from __future__ import annotations

import datetime
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
K = 10
N, VOCAB, NQ = 12_000, 400, 40


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup(rank, world, port, timeout_s):
    for p in (str(ROOT), str(ROOT / "go-fann_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _exact(data, qidx):
    """Exact filtered top-k ids and distances (uint8 L2, ties by id)."""
    import torch
    from gofann import workload_gpu as W
    ids = W.ground_truth(data, data["queries"], qidx, k=K)
    base = data["base"].to(torch.int64)
    qv = data["queries"].vectors.to(torch.int64)
    d = np.full(ids.shape, np.finfo(np.float32).max, np.float32)
    for j, qi in enumerate(qidx):
        ok = ids[j] != np.uint32(0xFFFFFFFF)
        if ok.any():
            rows = torch.from_numpy(ids[j][ok].astype(np.int64))
            d[j, ok] = (base[rows] - qv[qi]).square().sum(1).numpy().astype(np.float32)
    return ids, d


def _rank_main(rank, world, port, out_dir):
    import torch
    dist = _setup(rank, world, port, 60)
    from gofann import sharding as S, workload_gpu as W
    from oracle import oracle as O
    data = W.generate(device="cpu", seed=5, n=N, vocab=VOCAB, n_queries=NQ, max_tags=6, sel_lo=1e-3)
    lo, hi = S.shard_range(N, rank, world)
    shard = S.shard_data(data, lo, hi, "cpu")
    qidx = np.arange(NQ)
    ids, d = _exact(shard, qidx)
    ok = ids != np.uint32(0xFFFFFFFF)
    ids = np.where(ok, ids + np.uint32(lo), ids)  # gofann_offset_ids rule
    xchg = S.ShardExchange(world, NQ, K, "cpu")
    all_ids, all_d = xchg.gather(torch.from_numpy(ids.view(np.int32)), torch.from_numpy(d))
    if rank == 0:
        mi, md = O.shard_merge(all_ids.numpy().view(np.uint32), all_d.numpy(), K)
        gi, gd = _exact(data, qidx)
        np.savez(Path(out_dir) / "r0.npz", mi=mi, md=md, gi=gi, gd=gd, lo=np.array([lo, hi]))
    dist.barrier()
    dist.destroy_process_group()


def _rank_leaves(rank, world, port, out_dir):
    import torch
    dist = _setup(rank, world, port, 5)
    from gofann import sharding as S
    xchg = S.ShardExchange(world, 4, K, "cpu")
    if rank == 1:
        return  # leaves between steps: no exchange of its own in flight
    try:
        xchg.gather(torch.zeros((4, K), dtype=torch.int32), torch.zeros((4, K), dtype=torch.float32))
        (Path(out_dir) / "r0.txt").write_text("completed")
    except Exception as e:  # noqa: BLE001 - any backend error counts
        (Path(out_dir) / "r0.txt").write_text(f"error: {type(e).__name__}")


def _spawn(fn, tmp_path, world=2):
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=fn, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    return [p.exitcode for p in procs]


def test_shard_ranges_cover_the_base_set():
    sys.path.insert(0, str(ROOT / "go-fann_b200"))
    from gofann import sharding as S
    for n, world in [(10, 3), (7, 8), (10_000_000, 8), (1, 1)]:
        spans = [S.shard_range(n, r, world) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    with pytest.raises(ValueError):
        S.shard_range(10, 2, 2)


def test_two_rank_exchange_equals_global_topk(tmp_path):
    codes = _spawn(_rank_main, tmp_path)
    assert codes == [0, 0], codes
    r = np.load(tmp_path / "r0.npz")
    assert tuple(r["lo"]) == (0, N // 2)
    np.testing.assert_array_equal(r["mi"], r["gi"])
    np.testing.assert_array_equal(r["md"], r["gd"])
    assert (r["gi"] != np.uint32(0xFFFFFFFF)).any()


def test_rank_leaving_before_exchange_ends_peer_with_error(tmp_path):
    codes = _spawn(_rank_leaves, tmp_path)
    assert codes[1] == 0
    msg = (tmp_path / "r0.txt").read_text()
    assert msg.startswith("error"), msg
