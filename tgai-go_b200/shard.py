"""Host-side partitioning of the KV-cache path over ranks (one process per GPU).

Two ways to split the work, matching the two multi-GPU configurations:

* independent sequences (batched decode): whole sequences go to ranks; no
  data crosses ranks on the attention path.  `lpt_partition` balances the
  KV bytes (sum of context lengths) with the longest-processing-time greedy
  rule instead of equal sequence counts.
* one long sequence: the KV heads split into contiguous groups, one per rank,
  each rank owning its group's query heads (q head h reads KV head
  h * n_kv / n_heads, src/tgai_engine.c:3951); per-head outputs are then
  all-gathered so every rank holds the full [n_heads][head_dim] row.
"""
import heapq


def kv_head_shard(n_heads, n_kv_heads, world, rank):
    """Contiguous KV-head group of `rank`: (kv0, kv1, q0, q1) half-open ranges.

    Requires n_kv_heads % world == 0 and n_heads % n_kv_heads == 0, so each
    rank gets whole GQA groups."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if n_kv_heads % world or n_heads % n_kv_heads:
        raise ValueError(f"{n_kv_heads} KV heads / {n_heads} heads do not split over {world}")
    per = n_kv_heads // world
    group = n_heads // n_kv_heads
    kv0 = rank * per
    return kv0, kv0 + per, kv0 * group, (kv0 + per) * group


def lpt_partition(lengths, world):
    """Assign sequences to `world` ranks, longest first onto the least loaded
    rank.  Returns a list of index lists (each sorted ascending)."""
    heap = [(0, r) for r in range(world)]
    parts = [[] for _ in range(world)]
    for i in sorted(range(len(lengths)), key=lambda i: -int(lengths[i])):
        load, r = heapq.heappop(heap)
        parts[r].append(i)
        heapq.heappush(heap, (load + int(lengths[i]), r))
    return [sorted(p) for p in parts]


def gather_heads(local, world, group=None):
    """All-gather per-rank head outputs [..., heads_local, head_dim] into
    [..., heads_local*world, head_dim] in rank order (torch tensors; NCCL on
    GPUs, gloo on CPU)."""
    import torch
    import torch.distributed as dist
    if world == 1:
        return local
    local = local.contiguous()
    if dist.get_backend(group) == "nccl":
        buf = torch.empty((world,) + tuple(local.shape), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(buf, local, group=group)
    else:                                   # gloo has no single-tensor all-gather
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local, group=group)
        buf = torch.stack(parts)
    # [world, lead..., hl, hd] -> [lead..., world, hl, hd] -> [lead..., world*hl, hd]
    nd = local.dim()
    perm = list(range(1, nd - 1)) + [0, nd - 1, nd]
    out = buf.permute(*perm).contiguous()
    return out.reshape(*local.shape[:-2], world * local.shape[-2], local.shape[-1])


def max_over_ranks(value, world, device=None):
    """Max of a float over ranks (rank timing is the slowest rank's)."""
    if world == 1:
        return float(value)
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
