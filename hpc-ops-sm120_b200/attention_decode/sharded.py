"""Multi-GPU decode: one process per GPU, torch.distributed for the plumbing.

The reference is single-GPU; its only parallelism is the in-kernel split over
the sequence (csrc/decode.cu:197,206).  Two sharded modes sit on top of the
same kernels here:

* Batch / KV-head sharding (no communication): each rank owns whole
  sequences.  ``batch_shard`` gives contiguous equal slices;
  ``balance_by_tokens`` partitions variable-length sequences so every rank
  streams about the same number of KV bytes (greedy longest-first).
* Sequence sharding (very long contexts): rank r owns tokens
  ``token_shard(S, r, R)`` of every sequence.  Each rank computes its partial
  state (acc, m, l) per query head with ``attention_decode_partial``; the
  packed states (33,280 B per rank at Hq=64, D=128) are all-gathered over
  NCCL and merged by the same LSE combine kernel (``combine_partials``) on
  every rank, so the output is replicated.

The state packing and merge order are plain host logic and are covered on
CPU by gloo-rank tests.
"""

from __future__ import annotations

import heapq

import torch

from . import attention_decode_partial, combine_partials


def token_shard(length: int, rank: int, world: int) -> tuple[int, int]:
    """Token range [lo, hi) of `rank` when `length` tokens are split over `world` ranks."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    return length * rank // world, length * (rank + 1) // world


def batch_shard(batch: int, rank: int, world: int) -> slice:
    """Contiguous near-equal slice of the batch for `rank`."""
    lo, hi = token_shard(batch, rank, world)
    return slice(lo, hi)


def balance_by_tokens(lengths, world: int) -> list[list[int]]:
    """Assign sequences to ranks so the per-rank token sums are balanced
    (longest-processing-time-first greedy; ties broken by sequence index)."""
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    heap = [(0, r) for r in range(world)]
    parts: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        parts[r].append(i)
        heapq.heappush(heap, (load + int(lengths[i]), r))
    return [sorted(p) for p in parts]


def state_layout(rows: int, head_dim: int) -> tuple[int, int]:
    """(floats per packed state block, offset of the (m, l) pairs)."""
    return rows * (head_dim + 2), rows * head_dim


def unpack_gathered(gathered: torch.Tensor, world: int, rows: int, head_dim: int):
    """Views (acc [world, rows, D], ml [world, rows, 2]) into an all-gathered
    buffer of packed blocks [acc | ml] (part stride rows*(D+2) floats)."""
    block, ml_off = state_layout(rows, head_dim)
    g = gathered.view(world, block)
    return g[:, :ml_off].view(world, rows, head_dim), g[:, ml_off:].view(world, rows, 2)


class SequenceShardedDecode:
    """Callable decode step over a sequence-sharded KV cache.

    ``q`` is replicated on every rank; ``k_local``/``v_local`` hold this rank's
    token shard.  Buffers are allocated once, so the step can be captured in a
    CUDA graph together with its NCCL all_gather (``capture``) and replayed
    with one launch from the host; release the graph (``release``) before
    destroying the process group.  Eager steps are faster when steps run back
    to back (each decode kernel's programmatic launch overlaps the previous
    step's merge, which graph replays serialise); the graph helps when the
    host is the bottleneck."""

    def __init__(self, q, k_local, v_local, group=None, seqlens_local=None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.q, self.k, self.v, self.seqlens = q, k_local, v_local, seqlens_local
        batch, q_heads, _, head_dim = q.shape
        self.shape = q.shape
        self.rows, self.head_dim = batch * q_heads, head_dim
        block, ml_off = state_layout(self.rows, head_dim)
        self.buf = torch.empty(block, dtype=torch.float32, device=q.device)
        self.acc = self.buf[:ml_off].view(batch, q_heads, head_dim)
        self.ml = self.buf[ml_off:].view(batch, q_heads, 2)
        self.gathered = torch.empty(self.world * block, dtype=torch.float32, device=q.device)
        self.out = torch.empty((self.rows, head_dim), dtype=torch.bfloat16, device=q.device)
        self.graph = None

    def capture(self, warmup: int = 3):
        """Record one step (partial decode, all_gather, merge) reading
        ``self.q`` into a CUDA graph; ``__call__`` then replays it."""
        stream = torch.cuda.Stream(device=self.q.device)
        stream.wait_stream(torch.cuda.current_stream(self.q.device))
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                self.run(self.q)
        torch.cuda.current_stream(self.q.device).wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            self.run(self.q)
        self.graph = graph
        return self

    def run(self, q):
        attention_decode_partial(q, self.k, self.v, self.seqlens, out_acc=self.acc, out_ml=self.ml)
        self.dist.all_gather_into_tensor(self.gathered, self.buf, group=self.group)
        acc, ml = unpack_gathered(self.gathered, self.world, self.rows, self.head_dim)
        combine_partials(acc, ml, out=self.out)
        return self.out.view(self.shape)

    def __call__(self):
        """One step; the returned output buffer is reused by the next step."""
        if self.graph is not None:
            self.graph.replay()
            return self.out.view(self.shape)
        return self.run(self.q)

    def with_query(self, q):
        """A step reading ``q`` (copied into the captured query buffer when a
        graph is in use)."""
        if self.graph is None:
            return lambda: self.run(q)

        def step():
            self.q.copy_(q)
            return self()

        return step

    def release(self):
        """Drop the graph and the buffers (call before destroy_process_group)."""
        self.graph = None
        self.buf = self.gathered = self.out = None


def attention_decode_sequence_sharded(q, k_local, v_local, group=None, seqlens_local=None):
    """One sequence-sharded decode (allocates its buffers; see SequenceShardedDecode)."""
    return SequenceShardedDecode(q, k_local, v_local, group, seqlens_local)()
