"""Multi-rank host logic on CPU (gloo, world size 2): row sharding of a codebook linear
computed by the CPU oracle, the gather of the shards, the global Freivalds verdict, and
failure detection when a rank dies (the survivor's collective ends with an error within
the process-group timeout instead of hanging)."""

from __future__ import annotations

import datetime
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from int_model_approximation_b200 import sharding, synthetic


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, world: int, port: int, timeout_s: float = 60.0) -> None:
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _shard_worker(rank: int, world: int, port: int, result_dir: str) -> None:
    import oracle

    try:
        _init(rank, world, port)
        m, k, n = 37, 96, 40
        x = synthetic.student_t_activations(m, k, seed=1)
        w, ws = synthetic.normal_fp8_weights(n, k, seed=2)
        s, e = sharding.row_shard(m, world, rank)
        c_local, _y, out_local = oracle.codebook_linear(x[s:e], w, ws)
        c_full = sharding.all_gather_rows(c_local, m)
        out_full = sharding.all_gather_rows(out_local.view(torch.int16), m).view(torch.bfloat16)
        # Freivalds verdict: rank 1 corrupts one row of its shard
        a = oracle.fp8_codebook(oracle.per_token_fp8(x[s:e])[0])
        b = oracle.fp8_codebook(w).t().contiguous()
        r = torch.randint(1, 1 << 20, (n,), generator=torch.Generator().manual_seed(3))
        c_check = c_local.clone()
        if rank == 1:
            c_check[0, 0] += 1
        count = torch.tensor([oracle.freivalds_mismatch_rows(a, b, c_check, r)], dtype=torch.int64)
        sharding.global_mismatch(count)
        if rank == 0:
            c_ref, _y2, out_ref = oracle.codebook_linear(x, w, ws)
            ok = torch.equal(c_full, c_ref) and torch.equal(out_full.view(torch.int16), out_ref.view(torch.int16))
            with open(os.path.join(result_dir, "shard.txt"), "w") as f:
                f.write(f"{int(ok)} {int(count.item())}")
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001 - report to the parent
        with open(os.path.join(result_dir, f"error{rank}.txt"), "w") as f:
            f.write(traceback.format_exc())
        raise


def _dying_worker(rank: int, world: int, port: int, result_dir: str) -> None:
    _init(rank, world, port, timeout_s=3.0)
    if rank == 1:
        os._exit(0)   # leaves between steps, before the next collective
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        outcome = "completed"
    except Exception as exc:  # noqa: BLE001
        outcome = f"error: {type(exc).__name__}"
    with open(os.path.join(result_dir, "dying.txt"), "w") as f:
        f.write(outcome)


def test_row_and_column_shards_cover_everything():
    for total in (0, 1, 7, 512, 16384):
        for world in (1, 2, 3, 8):
            spans = [sharding.row_shard(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(e - s for s, e in spans) - min(e - s for s, e in spans) <= 1
    spans = [sharding.col_shard(18944, 8, r) for r in range(8)]
    assert spans[0][0] == 0 and spans[-1][1] == 18944
    assert all(s % 16 == 0 for s, _ in spans)
    with pytest.raises(ValueError):
        sharding.row_shard(10, 2, 2)


def test_two_gloo_ranks_shard_gather_and_verify(tmp_path):
    port = _free_port()
    mp.start_processes(_shard_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    errors = [p.read_text() for p in tmp_path.glob("error*.txt")]
    assert not errors, errors
    ok, count = (tmp_path / "shard.txt").read_text().split()
    assert ok == "1"
    assert count == "1"   # rank 1's corrupted row is the only rejected row, seen globally


def test_a_dead_rank_is_detected_by_the_survivor(tmp_path):
    port = _free_port()
    ctx = mp.start_processes(_dying_worker, args=(2, port, str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=120)
    for p in ctx.processes:
        if p.is_alive():
            p.kill()
    outcome = (tmp_path / "dying.txt").read_text()
    assert outcome.startswith("error"), outcome
