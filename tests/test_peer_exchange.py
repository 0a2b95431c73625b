"""Sequence sharding through exchange buffers on ONE GPU: the ranks of a
world are emulated in one process, each with its own exchange buffer, and
their steps run one after another on one stream (every rank's decode, then
every rank's merge), so no kernel waits on another one that runs at the same
time.  This checks the data path (states stored into every rank's slot, by
call parity), the flags and the device-side call counter, graph replay, and
that a merge whose peer never delivers gives up after its time limit with
an error status instead of hanging."""

from __future__ import annotations

import pytest
import torch

import attention_decode as ad
from attention_decode import _lib, sharded
from helpers import check, inputs, oracle_reference

pytestmark = pytest.mark.gpu


def _emulated_step(exchange, q, shards, outs, seqlens=None):
    for r, (k, v) in enumerate(shards):
        exchange.decode(q, k, v, rank=r, seqlens=None if seqlens is None else seqlens[r])
    for r in range(exchange.world):
        exchange.merge(outs[r], rank=r)


def _shard(k, v, world):
    S = k.shape[2]
    out = []
    for r in range(world):
        lo, hi = sharded.token_shard(S, r, world)
        out.append((k[:, :, lo:hi].contiguous(), v[:, :, lo:hi].contiguous()))
    return out


@pytest.mark.parametrize("world", (2, 3, 4, 8))
@pytest.mark.parametrize("length,dim,hq,hkv,batch", ((16384 + 37, 128, 64, 8, 1), (4099, 64, 32, 8, 2)))
def test_emulated_ranks_merge_to_full_decode(world, length, dim, hq, hkv, batch, device, record_property):
    q, k, v = inputs(device, length, dim, hkv, batch=batch, hq=hq, seed=301 + world)
    shards = _shard(k, v, world)
    rows = batch * hq
    exchange = sharded.PeerExchange.emulated(world, rows, dim, device)
    try:
        full = ad.attention_decode(q, k, v)
        expected = oracle_reference(q, k, v)
        for step in range(3):  # both parities, and a call counter that advances
            outs = [torch.full((rows, dim), float("nan"), dtype=torch.bfloat16, device=device) for _ in range(world)]
            _emulated_step(exchange, q, shards, outs)
            torch.cuda.synchronize(device)
            for r in range(world):
                got = outs[r].view(q.shape)
                check(got, expected, q, record_property, f"step{step}_rank{r}")
                check(got, full, q, None, atol=1e-2, rtol=2.0**-7)
        assert ad.read_error_flag(device.index or 0) == 0
    finally:
        exchange.close()


def test_emulated_ranks_with_sequence_lengths(device, record_property):
    world, batch, hq, hkv, dim, S = 4, 6, 32, 8, 128, 8192
    q, k, v = inputs(device, S, dim, hkv, batch=batch, hq=hq, seed=311)
    lengths = torch.tensor([8192, 1, 0, 5000, 2049, 6144], dtype=torch.int32, device=device)
    for b, n in enumerate(lengths.tolist()):
        k[b, :, n:] = float("nan")
        v[b, :, n:] = float("nan")
    shards = _shard(k, v, world)
    local_lens = []
    for r in range(world):
        lo, hi = sharded.token_shard(S, r, world)
        local_lens.append((lengths - lo).clamp(0, hi - lo).to(torch.int32))
    exchange = sharded.PeerExchange.emulated(world, batch * hq, dim, device)
    try:
        outs = [torch.empty((batch * hq, dim), dtype=torch.bfloat16, device=device) for _ in range(world)]
        _emulated_step(exchange, q, shards, outs, local_lens)
        torch.cuda.synchronize(device)
        expected = oracle_reference(q, k, v, lengths)
        for r in range(world):
            check(outs[r].view(q.shape), expected, q, record_property, f"rank{r}")
    finally:
        exchange.close()


def test_emulated_step_replays_from_a_graph(device, record_property):
    world, S, dim, hq, hkv = 2, 8192 + 5, 128, 64, 8
    q, k, v = inputs(device, S, dim, hkv, hq=hq, seed=321)
    q2 = inputs(device, 1, dim, hkv, hq=hq, seed=322)[0]
    shards = _shard(k, v, world)
    rows = hq
    exchange = sharded.PeerExchange.emulated(world, rows, dim, device)
    outs = [torch.empty((rows, dim), dtype=torch.bfloat16, device=device) for _ in range(world)]
    qbuf = q.clone()
    try:
        stream = torch.cuda.Stream(device=device)
        stream.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(stream):
            for _ in range(2):
                _emulated_step(exchange, qbuf, shards, outs)
        torch.cuda.current_stream(device).wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            _emulated_step(exchange, qbuf, shards, outs)
        for step, query in enumerate((q, q2, q, q2)):
            qbuf.copy_(query)
            graph.replay()
            torch.cuda.synchronize(device)
            expected = oracle_reference(query, k, v)
            for r in range(world):
                check(outs[r].view(q.shape), expected, query, record_property, f"replay{step}_rank{r}")
        del graph
        assert ad.read_error_flag(device.index or 0) == 0
    finally:
        exchange.close()


def test_missing_peer_ends_the_wait_with_an_error(device):
    """Rank 1 never decodes: rank 0's merge waits for a flag that nothing
    sets, gives up after its 20 ms limit, writes zero rows and sets the
    peer-timeout bit of the device error word; the context stays usable."""
    world, S, dim, hq, hkv = 2, 1024, 64, 32, 8
    q, k, v = inputs(device, S, dim, hkv, hq=hq, seed=331)
    shards = _shard(k, v, world)
    exchange = sharded.PeerExchange.emulated(world, hq, dim, device)
    try:
        ad.read_error_flag(device.index or 0)  # clear
        exchange.decode(q, *shards[0], rank=0)
        out = torch.full((hq, dim), 7.0, dtype=torch.bfloat16, device=device)
        exchange.merge(out, rank=0, timeout_s=0.02)
        torch.cuda.synchronize(device)
        flag = ad.read_error_flag(device.index or 0)
        assert flag & _lib.ADB_ERROR_FLAG_PEER_TIMEOUT
        assert torch.count_nonzero(out).item() == 0
        # the context still works
        full = ad.attention_decode(q, k, v)
        check(full, oracle_reference(q, k, v), q)
    finally:
        exchange.close()


def test_fused_merge_without_peers_times_out_with_error(device):
    """The fused decode + merge (adb_decode_exchange_merged) of rank 0 of a
    2-rank world whose rank 1 never runs: its merging CTAs wait for a flag
    that nothing sets, give up after the 20 ms limit, write zero rows and set
    the peer-timeout bit; the context stays usable.  (Only rank 0 launches,
    so no kernel waits on another one on this GPU.)"""
    import attention_decode

    world, S, dim, hq, hkv = 2, 1024, 64, 32, 8
    q, k, v = inputs(device, S, dim, hkv, hq=hq, seed=333)
    shards = _shard(k, v, world)
    exchange = sharded.PeerExchange.emulated(world, hq, dim, device)
    try:
        ad.read_error_flag(device.index or 0)  # clear
        out = torch.full((hq, dim), 7.0, dtype=torch.bfloat16, device=device)
        attention_decode._launch_exchange(q, *shards[0], None, exchange.bases, 0, out=out, timeout_us=20000)
        torch.cuda.synchronize(device)
        flag = ad.read_error_flag(device.index or 0)
        assert flag & _lib.ADB_ERROR_FLAG_PEER_TIMEOUT
        assert torch.count_nonzero(out).item() == 0
        full = ad.attention_decode(q, k, v)
        check(full, oracle_reference(q, k, v), q)
    finally:
        exchange.close()


def test_fused_merge_of_a_single_rank_equals_the_decode(device):
    """World of one: the fused launch publishes its own flag and merges its
    own state (no waiting on anything else), which must equal the plain
    decode."""
    import attention_decode

    S, dim, hq, hkv = 4099, 128, 64, 8
    q, k, v = inputs(device, S, dim, hkv, hq=hq, seed=334)
    exchange = sharded.PeerExchange.emulated(1, hq, dim, device)
    try:
        for _ in range(3):  # both parities
            out = torch.full((hq, dim), float("nan"), dtype=torch.bfloat16, device=device)
            attention_decode._launch_exchange(q, k, v, None, exchange.bases, 0, out=out, timeout_us=2_000_000)
            torch.cuda.synchronize(device)
            check(out.view(q.shape), oracle_reference(q, k, v), q)
        assert ad.read_error_flag(device.index or 0) == 0
    finally:
        exchange.close()
