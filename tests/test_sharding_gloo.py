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


def _presence_masks(fp8: torch.Tensor, pack_width: int) -> torch.Tensor:
    """CPU restatement of hawkeye_freivalds.class_presence: bit (c % 32) of word (c // 32)."""
    import oracle

    ids = oracle.class_ids(fp8)
    k = ids.shape[1]
    packs = max((k + pack_width - 1) // pack_width, 1)
    masks = torch.zeros((packs, 16), dtype=torch.int64)
    for p in range(packs):
        for c in torch.unique(ids[:, p * pack_width:(p + 1) * pack_width]).tolist():
            if c >= 0:
                masks[p, c // 32] |= 1 << (c % 32)
    return masks.to(torch.uint32).view(torch.int32) if hasattr(torch, "uint32") else masks.to(torch.int32)


def _popcount_rows(masks: torch.Tensor) -> list[int]:
    return [sum(bin(int(w) & 0xFFFFFFFF).count("1") for w in row) for row in masks.tolist()]


def _class_worker(rank: int, world: int, port: int, result_dir: str) -> None:
    import oracle
    from int_model_approximation_b200 import hawkeye_freivalds as hf

    try:
        _init(rank, world, port)
        x = synthetic.student_t_activations(29, 150, seed=4, outlier_fraction=0.05)
        xq, _ = oracle.per_token_fp8(x)
        w, _ = synthetic.normal_fp8_weights(9, 150, seed=5)
        s, e = sharding.row_shard(29, world, rank)
        width = 64   # 2 group lanes of 32
        glob = sharding.global_class_presence(_presence_masks(xq[s:e], width), None)
        full = _presence_masks(xq, width)
        stats = hf.class_count_stats(_popcount_rows(glob), _popcount_rows(_presence_masks(w, width)), 150,
                                     products_per_group=32, class_chunk=8, packed_count_lanes=6, packed_group_lanes=2)
        ref = oracle.class_count_stats(xq, w, class_chunk=8, packed_count_lanes=6, packed_group_lanes=2)
        # column-sharded Freivalds: partial vectors summed over ranks equal the unsharded ones
        r = torch.randint(0, 1 << 20, (9,), generator=torch.Generator().manual_seed(6))
        a = oracle.fp8_codebook(xq)
        b = oracle.fp8_codebook(w)
        c = oracle.int_gemm(a, b, b_is_nk=True)
        cs, ce = sharding.row_shard(9, world, rank)
        t_part = (b[cs:ce].t().to(torch.int64) @ r[cs:ce]).contiguous()
        cr_part = (c[:, cs:ce] @ r[cs:ce]).contiguous()
        sharding.combine_freivalds_partials(t_part)
        sharding.combine_freivalds_partials(cr_part)
        ok_check = torch.equal(a.to(torch.int64) @ t_part, cr_part)
        if rank == 0:
            with open(os.path.join(result_dir, "classes.txt"), "w") as f:
                f.write(f"{int(torch.equal(glob, full))} {int(stats.__dict__ == ref)} {int(ok_check)}")
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001 - report to the parent
        with open(os.path.join(result_dir, f"error{rank}.txt"), "w") as f:
            f.write(traceback.format_exc())
        raise


def test_two_gloo_ranks_share_class_lists_and_freivalds_partials(tmp_path):
    port = _free_port()
    mp.start_processes(_class_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    errors = [p.read_text() for p in tmp_path.glob("error*.txt")]
    assert not errors, errors
    assert (tmp_path / "classes.txt").read_text().split() == ["1", "1", "1"]
