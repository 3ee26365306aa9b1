"""Host logic of the N-sharded multi-GPU GEMM, run as 2 gloo ranks on CPU.

Each rank quantises the same seeded problem, keeps its column shard of the
weights and their scales (sharding.shard_bounds / shard_rows), computes its
block of C with the CPU oracle (standing in for the GPU kernel, which is
tested per shard by the GPU parity tests), and the blocks are all-gathered
(sharding.allgather_columns).  Rank 0 checks the assembled C bit-for-bit
against the unsharded oracle GEMM: column blocks are independent, so the
sharded result must be identical.
"""
import importlib
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, port, family, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        from oracle import oracle as orc
        sh = importlib.import_module("355_1_trans_b200.sharding")
        m, n, k = 48, 512, 256
        x = orc.normal((m, k), seed=11)
        w = orc.normal((n, k), seed=12)
        if family == "mxfp8":
            qa, sa = orc.quant_mxfp8(x)
            qb, sb = orc.quant_mxfp8(w)
            n0, n1 = sh.shard_bounds(n, WORLD, rank, 8)
            qb_s = sh.shard_rows(torch.from_numpy(qb), n0, n1).numpy()
            sb_s = sh.shard_rows(torch.from_numpy(sb), n0, n1).numpy()
            c_s = orc.gemm_mxfp8(qa, qb_s, sa, sb_s)
            full = orc.gemm_mxfp8(qa, qb, sa, sb) if rank == 0 else None
        else:
            qa, sa = orc.quant_fp8_block(x, 1)
            qb, sb = orc.quant_fp8_block(w, 128)
            n0, n1 = sh.shard_bounds(n, WORLD, rank, 128)
            qb_s = sh.shard_rows(torch.from_numpy(qb), n0, n1).numpy()
            sb_s = sh.shard_rows(torch.from_numpy(sb), n0, n1, rows_per_entry=128).numpy()
            c_s, _ = orc.gemm_fp8_block(qa, qb_s, sa, sb_s)
            full = orc.gemm_fp8_block(qa, qb, sa, sb)[0] if rank == 0 else None
        c = sh.allgather_columns(torch.from_numpy(np.ascontiguousarray(c_s)))
        if rank == 0:
            ok = c.shape == (m, n) and np.array_equal(c.numpy(), full)
            with open(result_path, "w") as f:
                f.write("ok" if ok else f"mismatch {tuple(c.shape)}")
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("family", ["mxfp8", "fp8block"])
def test_two_rank_column_sharding_is_exact(tmp_path, family):
    result = tmp_path / "result.txt"
    mp.start_processes(_rank_main, args=(_free_port(), family, str(result)), nprocs=WORLD, join=True,
                       start_method="spawn")
    assert result.read_text() == "ok"


def test_shard_bounds_cover_columns_once():
    sh = importlib.import_module("355_1_trans_b200.sharding")
    for n, world, gran in ((57344, 8, 128), (7168, 3, 128), (1000, 4, 8), (16, 8, 16)):
        spans = [sh.shard_bounds(n, world, r, gran) for r in range(world)]
        cols = np.zeros(n, np.int32)
        for n0, n1 in spans:
            assert n0 % gran == 0
            cols[n0:n1] += 1
        assert np.all(cols == 1), (n, world, gran)
    with pytest.raises(ValueError):
        sh.shard_bounds(128, 2, 2)


def _dead_peer_main(rank, port, result_path):
    """Rank 1 leaves right after joining; rank 0's gather must fail with an
    error (connection to the peer lost or the group timeout), not hang."""
    import time
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=10))
    if rank == 1:
        os._exit(0)   # dies between steps, no collective in flight
    sh = importlib.import_module("355_1_trans_b200.sharding")
    time.sleep(1.0)
    t0 = time.time()
    try:
        sh.allgather_columns(torch.zeros(4, 8))
        outcome = "no error"
    except Exception as e:   # noqa: BLE001 -- any collective failure is the expected outcome
        outcome = f"error after {time.time() - t0:.1f}s: {type(e).__name__}"
    with open(result_path, "w") as f:
        f.write(outcome)
    os._exit(0)


@pytest.mark.timeout(180)
def test_lost_rank_fails_fast(tmp_path):
    result = tmp_path / "result.txt"
    ctx = mp.start_processes(_dead_peer_main, args=(_free_port(), str(result)), nprocs=WORLD, join=False,
                             start_method="spawn")
    for p in ctx.processes:
        p.join(120)
    alive = [p for p in ctx.processes if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    text = result.read_text()
    assert text.startswith("error after"), text


@pytest.mark.parametrize("fam", ["mxfp4", "fp8block"])
def test_configs4_weights_are_the_same_for_every_rank_count(fam, monkeypatch):
    """bench.py's configs[4] record regenerates weight columns from per-block
    seeds on whichever rank needs them, and checks the gathered C against
    them: the concatenated shards of P ranks must be the very bytes of the
    unsharded matrix for P = 1, 2, 4, 8 (here on the CPU at a reduced size)."""
    import bench
    import bench_configs4 as c4
    monkeypatch.setattr(c4, "N", 4096)
    monkeypatch.setattr(c4, "K", 256)
    dev = torch.device("cpu")
    whole_q, whole_s = c4._weights(bench, fam, 0, 4096, dev)
    for p in (2, 4, 8):
        nl = 4096 // p
        parts = [c4._weights(bench, fam, r * nl, (r + 1) * nl, dev) for r in range(p)]
        assert torch.equal(torch.cat([q for q, _ in parts]), whole_q), (fam, p)
        assert torch.equal(torch.cat([s for _, s in parts]), whole_s), (fam, p)
    # a 128-column block regenerated alone (the parity check's unit) matches too
    q, s = c4._weights(bench, fam, 1664, 1792, dev)
    assert torch.equal(q, whole_q[1664:1792])
    assert torch.equal(s, whole_s[1664:1792] if fam == "mxfp4" else whole_s[13:14])
