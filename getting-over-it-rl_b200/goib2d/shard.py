"""Worlds sharded across GPUs (one process per GPU): contiguous world ranges, no communication on the step path,
one collective for per-world episode statistics.

Worlds are independent (nothing in b2World::Step reads another world), so the batch splits into contiguous ranges,
one per rank, each stepped by its own libgoib2d on its own GPU. Weak scaling: every rank owns `n_per_rank` worlds,
rank r worlds [r * n_per_rank, (r + 1) * n_per_rank) of the seeded workload (goib2d.configs draws each world from its
own generator, so a world's initial state does not depend on which rank builds it). The only collective is the
all-gather of per-world episode statistics at the end of an episode or a benchmark (NCCL over NVLink on the GPUs,
gloo in the CPU tests).
"""
import torch
import torch.distributed as dist


def world_range(n_per_rank, rank):
    """(first world, count) of a rank's shard."""
    return rank * n_per_rank, n_per_rank


def episode_stats(state, body, status=None):
    """Per-world statistics of one body: centre x, y and linear velocity x, y, plus the step's status word
    (float32 (N, 5)); `state` holds torch tensors (any device)."""
    c, v = state.bodies.c[:, body], state.bodies.v[:, body]
    n = c.shape[0]
    st = torch.zeros(n, dtype=torch.float32, device=c.device) if status is None else \
        torch.as_tensor(status, dtype=torch.float32, device=c.device)
    return torch.stack([c[:, 0], c[:, 1], v[:, 0], v[:, 1], st], 1).contiguous()


def gather_stats(stats):
    """All ranks' statistics in world order (every rank receives them). A single process returns its own."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return stats
    parts = [torch.empty_like(stats) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, stats.contiguous())
    return torch.cat(parts, 0)
