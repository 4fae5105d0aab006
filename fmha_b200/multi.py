"""Batch sharding across GPUs (one process per GPU, no collective).

Every (batch row, kv head) unit is independent, so N GPUs take N contiguous
batch ranges [B*r/N, B*(r+1)/N). Because the [B,H,S,D] layout is batch-major,
a shard is one contiguous slice of Q, K, V and O; the seeded generator is
indexed by the global element number, so a shard's inputs (and therefore its
outputs) are bit-identical to the same rows of a 1-GPU run. Outputs stay on
their GPU; gather_output() assembles them only for callers that ask.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    row0: int          # first global batch row
    rows: int          # rows in this shard
    q_offset: int      # element offsets of the shard inside the global tensors
    kv_offset: int
    o_offset: int


def shard_rows(batch: int, world: int, rank: int) -> tuple[int, int]:
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    return batch * rank // world, batch * (rank + 1) // world


def make_shard(batch, num_heads_q, num_heads_kv, seqlen_kv, head_dim, world, rank) -> Shard:
    lo, hi = shard_rows(batch, world, rank)
    return Shard(rank, world, lo, hi - lo, lo * num_heads_q * head_dim,
                 lo * num_heads_kv * seqlen_kv * head_dim, lo * num_heads_q * head_dim)


def gather_output(local_o, shard: Shard, group=None):
    """All-gather of the sharded O (flat fp16 or any dtype) into the full
    batch on every rank, through torch.distributed (NCCL over NVLink on GPUs,
    gloo on CPU). Shards may differ in size by one row."""
    import torch
    import torch.distributed as dist
    raw = local_o.reshape(-1).view(torch.uint8)  # bytes: every backend moves uint8
    n = torch.tensor([raw.numel()], dtype=torch.int64, device=raw.device)
    sizes = [torch.zeros_like(n) for _ in range(shard.world)]
    dist.all_gather(sizes, n, group=group)
    m = int(max(int(s.item()) for s in sizes))
    if all(int(s.item()) == m for s in sizes):
        # Equal shards: one collective straight into the output buffer.
        out = torch.empty(m * shard.world, dtype=torch.uint8, device=raw.device)
        dist.all_gather_into_tensor(out, raw.contiguous(), group=group)
        return out.view(local_o.dtype)
    buf = torch.zeros(m, dtype=torch.uint8, device=raw.device)
    buf[:raw.numel()] = raw
    parts = [torch.empty_like(buf) for _ in range(shard.world)]
    dist.all_gather(parts, buf, group=group)
    out = torch.cat([p[:int(s.item())] for p, s in zip(parts, sizes)])
    return out.view(local_o.dtype)


class ShardMonitor:
    """Host-side failure detection for the batch-sharded driver.

    Each rank posts its status for every step to a torch.distributed store
    (TCPStore; key "fmha/<step>/<rank>" = "ok" or "fail:<reason>") *between*
    steps, never while its kernels are in flight. ``wait_step`` collects the
    statuses of all ranks for a step with a bounded wait and returns the ranks
    that reported a failure and the ranks that never reported, so a driver can
    stop cleanly instead of blocking in a collective. Nothing here touches a
    GPU.
    """

    def __init__(self, store, rank: int, world: int, prefix: str = "fmha"):
        self.store, self.rank, self.world, self.prefix = store, rank, world, prefix

    def _key(self, step: int, rank: int) -> str:
        return f"{self.prefix}/{step}/{rank}"

    def report(self, step: int, ok: bool = True, reason: str = "") -> None:
        self.store.set(self._key(step, self.rank), "ok" if ok else f"fail:{reason}")

    def wait_step(self, step: int, timeout_s: float = 5.0, poll_s: float = 0.01):
        """Returns (failed: {rank: reason}, missing: [rank]) for ``step``."""
        import time
        deadline = time.monotonic() + timeout_s
        failed, seen = {}, set()
        while True:
            for r in range(self.world):
                if r in seen:
                    continue
                key = self._key(step, r)
                if self.store.check([key]):
                    v = self.store.get(key).decode()
                    seen.add(r)
                    if v != "ok":
                        failed[r] = v[len("fail:"):]
            if len(seen) == self.world or time.monotonic() >= deadline:
                break
            time.sleep(poll_s)
        missing = [r for r in range(self.world) if r not in seen]
        return failed, missing
