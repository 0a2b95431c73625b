"""Multi-GPU decode: one process per GPU, torch.distributed for the plumbing.

The reference is single-GPU; its only parallelism is the in-kernel split over
the sequence (csrc/decode.cu:197,206).  Two sharded modes sit on top of the
same kernels here:

* Batch / KV-head sharding (no communication): each rank owns whole
  sequences.  ``batch_shard`` gives contiguous equal slices;
  ``balance_by_tokens`` partitions variable-length sequences so every rank
  streams about the same number of KV bytes (greedy longest-first).
* Sequence sharding (very long contexts): rank r owns tokens
  ``token_shard(S, r, R)`` of every sequence and computes its partial state
  (acc, m, l) per query head; the states (33,280 B per rank at Hq=64,
  D=128) of all ranks are merged on every rank, so the output is
  replicated.  Two transports:

  - ``"p2p"`` (default): the decode kernel itself stores its states into
    every rank's exchange buffer over NVLink (peer memory mapped with CUDA
    IPC) and raises a flag there; a small merge kernel waits for the flags
    and merges.  Two launches per step, no collective library call.
  - ``"nccl"``: ``attention_decode_partial``, an NCCL all_gather of the
    packed states, then ``combine_partials``.

The state packing and merge order are plain host logic and are covered on
CPU by gloo-rank tests.
"""

from __future__ import annotations

import ctypes
import heapq
import socket

import torch

from . import _launch_exchange, _lib, attention_decode_partial, combine_partials

DEFAULT_PEER_TIMEOUT_S = 2.0


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


class PeerExchange:
    """Exchange buffers of a sequence-sharded decode over NVLink peer memory.

    Collective: every rank of `group` constructs it with the same `rows`
    (= batch * q_heads) and `head_dim`.  Each rank allocates one zeroed
    buffer in its own HBM (adb_exchange_alloc), the CUDA IPC handles are
    all-gathered over `group`, and each rank maps the other ranks' buffers;
    ``bases[r]`` is rank r's buffer as seen from this process.  ``close``
    (also collective) unmaps and frees after every rank's work is done."""

    def __init__(self, rows: int, head_dim: int, group=None, device=None, *, _world=None):
        self.lib = _lib.load_library()
        self.rows, self.head_dim = int(rows), int(head_dim)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.group = group
        self._own: list[int] = []
        self._mapped: list[int] = []
        if _world is not None:  # single-process emulation (see `emulated`)
            self.dist, self.world, self.rank = None, _world, None
            self.bases = [self._alloc() for _ in range(_world)]
            self.fused = False  # the emulated ranks share one GPU
            return
        import torch.distributed as dist

        self.dist = dist
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        mine = self._alloc()
        handle = ctypes.create_string_buffer(_lib.ADB_IPC_HANDLE_BYTES)
        _lib.check(self.lib, self.lib.adb_ipc_handle(mine, self.index, handle))
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        # The fused step (decode and merge in one launch) makes each rank's
        # kernel wait for the others' kernels, so it is used only when every
        # rank has a GPU of its own.
        props = torch.cuda.get_device_properties(self.device)
        where = (socket.gethostname(), props.pci_domain_id, props.pci_bus_id, props.pci_device_id)
        places = [None] * self.world
        dist.all_gather_object(places, where, group=group)
        self.fused = len(set(places)) == self.world
        self.bases = []
        for r, raw in enumerate(handles):
            if r == self.rank:
                self.bases.append(mine)
                continue
            ptr = ctypes.c_void_p()
            _lib.check(self.lib, self.lib.adb_ipc_open(raw, self.index, ctypes.byref(ptr)))
            self._mapped.append(ptr.value)
            self.bases.append(ptr.value)
        dist.barrier(group=group)

    @classmethod
    def emulated(cls, world: int, rows: int, head_dim: int, device=None) -> "PeerExchange":
        """`world` buffers on one GPU in one process, for driving the ranks'
        steps one after another (tests of the data path and the flags)."""
        return cls(rows, head_dim, device=device, _world=world)

    def _alloc(self) -> int:
        size = ctypes.c_size_t(0)
        _lib.check(self.lib, self.lib.adb_exchange_size(self.rows, self.head_dim, self.world, ctypes.byref(size)))
        ptr = ctypes.c_void_p()
        _lib.check(self.lib, self.lib.adb_exchange_alloc(size.value, self.index, ctypes.byref(ptr)))
        self._own.append(ptr.value)
        return ptr.value

    def decode(self, q, k, v, rank: int | None = None, seqlens=None):
        """This rank's partial decode; its states go to every rank's buffer."""
        _launch_exchange(q, k, v, seqlens, self.bases, self.rank if rank is None else rank)

    def decode_merged(self, q, k, v, out, seqlens=None, timeout_s: float = DEFAULT_PEER_TIMEOUT_S):
        """decode + merge in one launch (adb_decode_exchange_merged): this
        rank's states go to every buffer and the merged rows to `out`.  Only
        when ``self.fused`` (every rank on its own GPU)."""
        if not self.fused:
            raise RuntimeError("decode_merged needs every rank on a GPU of its own (use decode + merge)")
        if out.dtype != torch.bfloat16 or not out.is_contiguous() or out.numel() != self.rows * self.head_dim:
            raise ValueError("out must be a contiguous bf16 buffer of rows * head_dim elements")
        _launch_exchange(q, k, v, seqlens, self.bases, self.rank, out=out, timeout_us=max(1, int(timeout_s * 1e6)))
        return out

    def merge(self, out, rank: int | None = None, timeout_s: float = DEFAULT_PEER_TIMEOUT_S):
        """Wait for every rank's states of this call (bounded) and merge them
        into `out` (contiguous BF16, rows * head_dim elements)."""
        if out.dtype != torch.bfloat16 or not out.is_contiguous() or out.numel() != self.rows * self.head_dim:
            raise ValueError("out must be a contiguous bf16 buffer of rows * head_dim elements")
        r = self.rank if rank is None else rank
        stream = torch._C._cuda_getCurrentRawStream(self.index)
        _lib.check(
            self.lib,
            self.lib.adb_exchange_merge(
                self.bases[r], self.world, self.rows, self.head_dim, out.data_ptr(),
                max(1, int(timeout_s * 1e6)), self.index, stream,
            ),
        )
        return out

    def close(self):
        """Unmap the peers' buffers and free this rank's (collective)."""
        if self.bases is None:
            return
        torch.cuda.synchronize(self.device)
        if self.dist is not None:
            self.dist.barrier(group=self.group)
        for ptr in self._mapped:
            _lib.check(self.lib, self.lib.adb_ipc_close(ptr, self.index))
        for ptr in self._own:
            _lib.check(self.lib, self.lib.adb_exchange_free(ptr, self.index))
        self._mapped, self._own, self.bases = [], [], None


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

    def __init__(self, q, k_local, v_local, group=None, seqlens_local=None, transport: str = "p2p",
                 timeout_s: float = DEFAULT_PEER_TIMEOUT_S, fused: bool | None = None):
        import torch.distributed as dist

        if transport not in ("p2p", "nccl"):
            raise ValueError(f"unknown transport {transport!r} (expected 'p2p' or 'nccl')")
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.transport = transport
        self.timeout_s = timeout_s
        self.q, self.k, self.v, self.seqlens = q, k_local, v_local, seqlens_local
        batch, q_heads, _, head_dim = q.shape
        self.shape = q.shape
        self.rows, self.head_dim = batch * q_heads, head_dim
        self.out = torch.empty((self.rows, head_dim), dtype=torch.bfloat16, device=q.device)
        self.graph = None
        self.exchange = None
        self.buf = self.gathered = None
        self.fused = False
        if transport == "p2p":
            self.exchange = PeerExchange(self.rows, head_dim, group, q.device)
            self.fused = self.exchange.fused if fused is None else (bool(fused) and self.exchange.fused)
            return
        block, ml_off = state_layout(self.rows, head_dim)
        self.buf = torch.empty(block, dtype=torch.float32, device=q.device)
        self.acc = self.buf[:ml_off].view(batch, q_heads, head_dim)
        self.ml = self.buf[ml_off:].view(batch, q_heads, 2)
        self.gathered = torch.empty(self.world * block, dtype=torch.float32, device=q.device)

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
        if self.exchange is not None:
            if self.fused:
                self.exchange.decode_merged(q, self.k, self.v, self.out, seqlens=self.seqlens, timeout_s=self.timeout_s)
            else:
                self.exchange.decode(q, self.k, self.v, seqlens=self.seqlens)
                self.exchange.merge(self.out, timeout_s=self.timeout_s)
            return self.out.view(self.shape)
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
        """Drop the graph and the buffers (collective; call on every rank
        before destroy_process_group)."""
        self.graph = None
        if self.exchange is not None:
            self.exchange.close()
            self.exchange = None
        self.buf = self.gathered = self.out = None


def attention_decode_sequence_sharded(q, k_local, v_local, group=None, seqlens_local=None, transport="p2p"):
    """One sequence-sharded decode (sets up and releases its buffers; see
    SequenceShardedDecode).  Returns a new output tensor."""
    step = SequenceShardedDecode(q, k_local, v_local, group, seqlens_local, transport=transport)
    try:
        return step().clone()
    finally:
        step.release()


# The name the sequence-sharded entry point is planned under.
attention_decode_sharded = attention_decode_sequence_sharded
