"""Host logic of the multi-GPU token sharding, tested with gloo ranks on CPU."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from probe_b200.sharding import gather_rows, local_segments, shard_rows, shard_segments


def test_shard_rows_cover_exactly():
    for total in (0, 1, 7, 32760, 4095):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_rows(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            for (a0, b0), (a1, b1) in zip(spans, spans[1:]):
                assert b0 == a1
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    assert shard_rows(32760, 8, 7) == (28665, 32760)
    with pytest.raises(ValueError):
        shard_rows(10, 2, 2)


def test_shard_segments_whole_and_balanced():
    seg = [0, 100, 150, 151, 400, 1000, 1024]
    for world in (1, 2, 3, 4, 8):
        groups = shard_segments(seg, world)
        assert len(groups) == world
        assert groups[0][0] == 0 and groups[-1][1] == len(seg) - 1
        for (a0, b0), (a1, b1) in zip(groups, groups[1:]):
            assert b0 == a1
    g2 = shard_segments(seg, 2)
    assert g2 == [(0, 4), (4, 6)]  # split at token 400 (closest boundary to 512)
    st = torch.tensor(seg)
    ad = torch.arange(6)
    t0, t1, ls, la = local_segments(st, ad, 2, 1)
    assert (t0, t1) == (400, 1024)
    assert ls.tolist() == [0, 600, 624] and la.tolist() == [4, 5]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        from datetime import timedelta

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
        n = 5
        verdict = "ok"
        for total in (37, 36):  # uneven shards (padded gather), then equal ones (straight into the output)
            a, b = shard_rows(total, world, rank)
            local = torch.arange(a, b, dtype=torch.float32)[:, None].repeat(1, n) * 10 + torch.arange(n)
            if mode == "fail" and rank == 1:
                raise RuntimeError("injected failure before the all-gather")
            out = torch.full((total, n), -1.0) if total == 36 else None
            full = gather_rows(local, total, out=out)
            want = torch.arange(total, dtype=torch.float32)[:, None].repeat(1, n) * 10 + torch.arange(n)
            if not torch.equal(full, want) or (out is not None and full.data_ptr() != out.data_ptr()):
                verdict = "mismatch"
        q.put((rank, verdict))
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001
        q.put((rank, f"error: {type(exc).__name__}: {str(exc)[:80]}"))


def _run(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    for p in procs:
        if p.is_alive():
            p.kill()
    res = {}
    while not q.empty():
        r, v = q.get()
        res[r] = v
    return res


def test_gather_rows_gloo_two_ranks():
    res = _run(2, "ok")
    assert res == {0: "ok", 1: "ok"}, res


def test_injected_rank_failure_is_reported_not_hung():
    """Rank 1 raises before the all-gather; rank 0's collective ends with an error
    within the process-group timeout instead of hanging."""
    res = _run(2, "fail")
    assert res[1].startswith("error: RuntimeError: injected failure"), res
    assert res[0].startswith("error"), res
