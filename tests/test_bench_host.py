"""Host-side logic of bench.py (CPU): the L2-defeating input rotation keeps a
rank's batch slice, so strong-scaling steps decode only that rank's share."""

from __future__ import annotations

import importlib.util
import os

import torch

from attention_decode import sharded
from attention_decode.workloads import BaselineConfig

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def load_bench():
    spec = importlib.util.spec_from_file_location("bench_module", os.path.join(ROOT, "bench.py"))
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def test_rotation_sets_keep_the_rank_slice():
    bench = load_bench()
    cfg = BaselineConfig("tiny", 8, 8, 2, 64, 256)
    world = 4
    for rank in range(world):
        rows = list(range(cfg.batch))[sharded.batch_shard(cfg.batch, rank, world)]
        q, k, v, _ = cfg.make_inputs("cpu", seed=11, batch_slice=rows)
        sets, kv_bytes = bench.rotation_sets(cfg, "cpu", 11 + 1009 * rank, (q, k, v), rows)
        assert kv_bytes == 2 * k.numel() * k.element_size()
        assert len(sets) > 1  # far below twice the L2: the steps rotate
        for qi, ki, vi in sets:
            assert qi.shape == q.shape and ki.shape == k.shape and vi.shape == v.shape
        assert not torch.equal(sets[0][1], sets[1][1])  # independent sets


def test_rotation_sets_whole_batch_by_default():
    bench = load_bench()
    cfg = BaselineConfig("tiny", 2, 4, 1, 64, 128)
    q, k, v, _ = cfg.make_inputs("cpu", seed=3)
    sets, _ = bench.rotation_sets(cfg, "cpu", 3, (q, k, v))
    assert all(ki.shape == k.shape for _, ki, _ in sets)
