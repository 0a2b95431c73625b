"""Multi-GPU decode: sequence sharding (partial states exchanged through
NVLink peer memory by the decode kernel itself -- merged in the same launch,
or by a second kernel -- and through an NCCL all_gather; merged on every
rank, eagerly and replayed from a CUDA graph) and
batch sharding (no collective), over 2, 4 and 8 ranks as far as the GPUs
go (one GPU per rank).  Ranks are spawned
processes, one per GPU, with a short process-group timeout so that a failure
ends in an error, not a hang."""

from __future__ import annotations

import os
import socket
import traceback
from datetime import timedelta

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        import attention_decode as ad
        from attention_decode import sharded
        from helpers import check, inputs, oracle_reference

        device = torch.device("cuda", rank)
        torch.cuda.set_device(device)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                                device_id=device)
        # --- sequence sharding: B=1, Hq=64, Hkv=8 (group 8), S=16384+37
        S = 16384 + 37
        q, k, v = inputs(device, S, 128, 8, batch=1, hq=64, seed=91)  # same values on every rank
        lo, hi = sharded.token_shard(S, rank, world)
        full = ad.attention_decode(q, k, v)
        expected = oracle_reference(q, k, v) if rank == 0 else None
        q2 = inputs(device, 1, 128, 8, batch=1, hq=64, seed=93)[0]
        full2 = ad.attention_decode(q2, k, v)
        # p2p fused (decode and merge in one launch, the default on distinct
        # GPUs), p2p in two launches, and NCCL
        for transport, fused in (("p2p", None), ("p2p", False), ("nccl", None)):
            step = sharded.SequenceShardedDecode(
                q.clone(), k[:, :, lo:hi].contiguous(), v[:, :, lo:hi].contiguous(), transport=transport,
                fused=fused,
            )
            if transport == "p2p":
                assert step.fused == (fused is None)
            out = step().clone()
            again = step().clone()
            torch.cuda.synchronize(device)
            check(out, full, q, atol=1e-2, rtol=2.0**-7)
            check(again, out, q, atol=1e-3, rtol=2.0**-7)
            if expected is not None:
                check(out, expected, q)
            for _ in range(5):  # back to back, no host synchronisation between steps
                step()
            check(step.with_query(q2)().clone(), full2, q2, atol=1e-2, rtol=2.0**-7)
            graphed = step.capture()
            for query, want in ((q, full), (q2, full2), (q, full)):
                check(graphed.with_query(query)().clone(), want, query, atol=1e-2, rtol=2.0**-7)
            step.release()
        assert ad.read_error_flag(rank) == 0
        # --- batch sharding: each rank decodes its slice of an 8-sequence batch
        q, k, v = inputs(device, 3000, 128, 8, batch=8, hq=32, seed=92)
        sl = sharded.batch_shard(8, rank, world)
        mine = ad.attention_decode(q[sl].contiguous(), k[sl].contiguous(), v[sl].contiguous())
        check(mine, ad.attention_decode(q, k, v)[sl], q[sl], atol=1e-2, rtol=2.0**-7)
        dist.barrier()
        results.put((rank, "ok", None))
    except Exception:
        results.put((rank, "error", traceback.format_exc()))
    finally:
        try:
            import torch.distributed as dist

            if dist.is_initialized():
                dist.destroy_process_group()
        except Exception:
            pass


@pytest.mark.parametrize("world", (2, 4, 8))
def test_sequence_and_batch_sharding_over_nccl(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            rank, status, payload = results.get(timeout=300)
            out[rank] = (status, payload)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank in range(world):
        assert out[rank][0] == "ok", out[rank][1]
