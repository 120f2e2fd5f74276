"""Two-GPU check of the row-parallel all-reduce fused into the decode GEMV
(tf_w4a16_linear_allreduce through tokenforge_b200.tp.PeerMailbox), against the same shard run
through the plain GEMV plus an NCCL all-reduce and against the oracle's fp64 product of the
unsharded layer. Runs as two spawned child processes (one per GPU, NCCL with NVLS off); skipped
on machines with fewer than two GPUs."""

from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2
SHAPES = [(3584, 3584), (3584, 18944)]  # Qwen2.5-7B o and down: N, K
MS = [1, 3, 8]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return int(s.getsockname()[1])


def _rank_main(rank: int, port: int, out: dict) -> None:  # type: ignore[type-arg]
    import datetime

    import torch.distributed as dist

    from tests.numerics import cases
    from tokenforge_b200 import tp

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, device_id=device,
                            timeout=datetime.timedelta(seconds=60))
    peers = tp.PeerMailbox(max_m=8, max_n=4096, device=device)
    try:
        for n, k in SHAPES:
            w = cases.layer_weights(n, k, 3)
            b = cases.bias(n, 3)
            shard = tp.shard_layer(w.to(device), "row", rank, WORLD, b.to(device))
            for m in MS:
                x = cases.activations(m, k, m).to(device)
                torch.cuda.synchronize(device)
                dist.barrier()  # peers must reach each fused call within the kernel's 2 s wait
                fused = [tp.linear_shard(x, shard, peers=peers) for _ in range(3)]
                plain = tp.linear_shard(x, shard)
                # Graph capture of two fused calls (the mailbox counts calls on the device).
                s = torch.cuda.Stream(device)
                s.wait_stream(torch.cuda.current_stream(device))
                with torch.cuda.stream(s):
                    tp.linear_shard(x, shard, peers=peers)
                torch.cuda.current_stream(device).wait_stream(s)
                torch.cuda.synchronize(device)
                dist.barrier()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    g1 = tp.linear_shard(x, shard, peers=peers)
                    g2 = tp.linear_shard(x, shard, peers=peers)
                replays = []
                for _ in range(3):
                    g.replay()
                    torch.cuda.synchronize(device)
                    replays.append((g1.clone(), g2.clone()))
                del g
                torch.cuda.synchronize(device)
                gathered = [torch.empty_like(fused[0]) for _ in range(WORLD)]
                dist.all_gather(gathered, fused[0])
                if rank == 0:
                    out[(n, k, m)] = {
                        "fused": [f.cpu() for f in fused],
                        "plain": plain.cpu(),
                        "ranks": [t.cpu() for t in gathered],
                        "replays": [(a.cpu(), c.cpu()) for a, c in replays],
                    }
        errs: list[object] = [None] * WORLD
        dist.all_gather_object(errs, peers.error())
        if rank == 0:
            out["error"] = errs
    finally:
        peers.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs two GPUs")
def test_fused_row_parallel_allreduce_two_gpus() -> None:
    import torch.multiprocessing as mp

    from oracle import oracle
    from tests.numerics import cases
    from tests.numerics.tolerance import atol

    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_rank_main, args=(_free_port(), out), nprocs=WORLD,
                           start_method="spawn")
        res = dict(out)
    assert res["error"] == [0] * WORLD, f"a peer wait timed out: {res['error']}"
    for n, k in SHAPES:
        w = cases.layer_weights(n, k, 3)
        b = cases.bias(n, 3)
        w16 = oracle.dequantize_tf(w.qweight_t, w.scales, w.qzeros, w.group_size)
        for m in MS:
            r = res[(n, k, m)]
            x = cases.activations(m, k, m)
            ref = oracle.w4a16_reference(x, w.qweight_t, w.scales, w.qzeros, w.group_size, b)
            tol = atol(x, w16, "cuda")
            first = r["fused"][0]
            for again in r["fused"][1:]:
                assert torch.equal(again, first), "fused result changed between calls"
            for rk in r["ranks"]:
                assert torch.equal(rk, first), "ranks disagree"
            for g1, g2 in r["replays"]:
                assert torch.equal(g1, first) and torch.equal(g2, first), "graph replay differs"
            err = float((first.double() - ref).abs().max())
            assert err <= tol, f"fused (m={m}, k={k}): {err:.3e} > {tol:.3e}"
            err_plain = float((r["plain"].double() - ref).abs().max())
            assert err_plain <= 2 * tol, f"NCCL path (m={m}, k={k}): {err_plain:.3e}"
