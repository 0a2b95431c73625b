"""Host logic of the multi-GPU modes on CPU ranks (gloo, world size 2).

The partial states come from the CPU oracle, so no GPU is involved: these
tests check the token/batch partitioning, the packed state layout that is
all-gathered between ranks, its unpacking, the merge order, and that a failing
rank surfaces as an error on the others within the process-group timeout.
"""

from __future__ import annotations

import os
import socket
import sys
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from attention_decode import sharded
from oracle import attention_decode_oracle as oracle


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
        if mode == "sequence":
            rng = np.random.default_rng(5)
            B, Hq, Hkv, S, D = 2, 16, 4, 1001, 64
            q = oracle.f32_to_bf16_bits(rng.standard_normal((B, Hq, 1, D), dtype=np.float32))
            k = oracle.f32_to_bf16_bits(rng.standard_normal((B, Hkv, S, D), dtype=np.float32))
            v = oracle.f32_to_bf16_bits(rng.standard_normal((B, Hkv, S, D), dtype=np.float32))
            lo, hi = sharded.token_shard(S, rank, world)
            acc, m, l = oracle.partial_state(q, k, v, lo, hi)
            rows = B * Hq
            block, ml_off = sharded.state_layout(rows, D)
            packed = torch.empty(block, dtype=torch.float32)
            packed[:ml_off] = torch.from_numpy(acc.reshape(-1))
            packed[ml_off:] = torch.from_numpy(np.stack([m.reshape(-1), l.reshape(-1)], -1).reshape(-1))
            parts = [torch.empty(block, dtype=torch.float32) for _ in range(world)]
            dist.all_gather(parts, packed)
            gathered = torch.cat(parts)
            acc_v, ml_v = sharded.unpack_gathered(gathered, world, rows, D)
            assert acc_v.shape == (world, rows, D) and ml_v.shape == (world, rows, 2)
            assert acc_v.stride(0) == block and ml_v.stride(0) == block
            merged = oracle.merge_states(acc_v.numpy(), ml_v[..., 0].numpy(), ml_v[..., 1].numpy())
            full = oracle.reference_fp32(q, k, v).reshape(rows, D)
            err = float(np.abs(merged - full).max())
            results.put((rank, "ok", err))
        elif mode == "fail":
            if rank == 1:
                raise RuntimeError("injected failure on rank 1")
            t = torch.ones(4)
            dist.all_reduce(t)  # rank 1 never joins: must time out, not hang
            results.put((rank, "no-error", None))
    except Exception as exc:  # reported to the parent
        results.put((rank, "error", f"{type(exc).__name__}: {exc}"))
    finally:
        try:
            if dist.is_initialized():
                dist.destroy_process_group()
        except Exception:
            traceback.print_exc()


def _run(mode, world=2, timeout=60):
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, results)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        rank, status, payload = results.get(timeout=timeout)
        out[rank] = (status, payload)
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return out


def test_sequence_sharded_states_merge_to_full_attention():
    out = _run("sequence")
    for rank in (0, 1):
        status, err = out[rank]
        assert status == "ok", err
        assert err < 1e-4


def test_failing_rank_surfaces_as_error_within_timeout():
    out = _run("fail")
    assert out[1][0] == "error" and "injected" in out[1][1]
    assert out[0][0] == "error"  # the collective ended with an error, not a hang


@pytest.mark.parametrize("length,world", [(131072, 8), (4097, 3), (5, 8), (1, 2)])
def test_token_shards_partition_the_sequence(length, world):
    bounds = [sharded.token_shard(length, r, world) for r in range(world)]
    assert bounds[0][0] == 0 and bounds[-1][1] == length
    for (a, b), (c, d) in zip(bounds, bounds[1:]):
        assert b == c and a <= b
    sizes = [b - a for a, b in bounds]
    assert max(sizes) - min(sizes) <= 1


def test_balance_by_tokens_is_a_partition_and_balanced():
    rng = np.random.default_rng(3)
    lengths = rng.integers(1, 8193, 64).tolist()
    for world in (1, 2, 4, 8):
        parts = sharded.balance_by_tokens(lengths, world)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(64))
        loads = [sum(lengths[i] for i in p) for p in parts]
        assert max(loads) - min(loads) <= max(lengths)


def test_batch_shard_slices_cover_the_batch():
    for batch, world in [(128, 8), (32, 3), (1, 2)]:
        slices = [sharded.batch_shard(batch, r, world) for r in range(world)]
        covered = [i for s in slices for i in range(batch)[s]]
        assert covered == list(range(batch))


def test_batch_shards_of_baseline_inputs_reproduce_the_full_batch():
    """A rank's share of one global batch (slice or token-balanced index list)
    holds exactly the full batch's rows, so strong scaling shards one problem."""
    from attention_decode.workloads import BaselineConfig

    cfg = BaselineConfig("small", 6, 8, 2, 64, 40, varlen=True, extreme=True)
    q, k, v, lens = cfg.make_inputs("cpu", seed=11)
    parts = sharded.balance_by_tokens(lens.tolist(), 3)
    for part in parts + [list(range(6))[sharded.batch_shard(6, 1, 3)]]:
        qs, ks, vs, ls = cfg.make_inputs("cpu", seed=11, batch_slice=part)
        assert torch.equal(qs, q[part]) and torch.equal(ks, k[part]) and torch.equal(vs, v[part])
        assert torch.equal(ls, lens[part])


if __name__ == "__main__":
    sys.exit(pytest.main([__file__, "-q"]))
