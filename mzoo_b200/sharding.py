"""Work partitioning of the hot path across the GPUs of one node (one process per GPU).

Every unit of this path is independent: decode sequences, prefill query
tokens, indexer query blocks and training batch elements need nothing from each other, so
there is no data-path collective.  The one collective is an optional output gather, done
with ``torch.distributed.all_gather_into_tensor`` (NCCL over NVLink on GPUs, gloo on CPU).

- ``shard_sequences`` -- decode: greedy longest-first by context length (the indexer's key
  stream dominates a decode step and grows with the context).
- ``shard_tokens`` -- prefill: cyclic chunks of query tokens so every rank gets the same mix
  of early (cheap, short causal range) and late (expensive) tokens.
- ``gather_rows`` -- pad each rank's rows to a common count, all-gather, then undo the
  assignment so row i of the result is unit i.
"""

import torch


def shard_sequences(lens, world: int) -> list:
    """Assign sequences to ``world`` ranks, longest first, each to the least-loaded rank
    (load = summed context length).  Returns the ascending sequence ids of every rank."""
    order = sorted(range(len(lens)), key=lambda b: (-int(lens[b]), b))
    load = [0] * world
    owned = [[] for _ in range(world)]
    for b in order:
        r = min(range(world), key=lambda i: (load[i], i))
        owned[r].append(b)
        load[r] += int(lens[b])
    return [sorted(o) for o in owned]


def shard_tokens(n_tokens: int, world: int, chunk: int = 128) -> list:
    """Cyclic assignment of ``chunk``-token blocks: rank r gets blocks r, r + world, ...
    Returns the token ids of every rank (ascending)."""
    out = [[] for _ in range(world)]
    for blk, t0 in enumerate(range(0, n_tokens, chunk)):
        out[blk % world].extend(range(t0, min(n_tokens, t0 + chunk)))
    return out


def gather_rows(local: torch.Tensor, owned: list, world_owned: list, group=None) -> torch.Tensor:
    """All-gather per-rank rows (``local[i]`` is unit ``owned[i]``) into one tensor indexed
    by unit id.  ``world_owned`` is every rank's ``owned`` list (the same on all ranks)."""
    import torch.distributed as dist
    world = len(world_owned)
    width = max(len(o) for o in world_owned)
    pad = local.new_zeros((width,) + tuple(local.shape[1:]))
    pad[:len(owned)] = local
    buf = local.new_empty((world * width,) + tuple(local.shape[1:]))
    dist.all_gather_into_tensor(buf, pad, group=group)
    n = sum(len(o) for o in world_owned)
    out = local.new_empty((n,) + tuple(local.shape[1:]))
    for r, o in enumerate(world_owned):
        if o:
            out[torch.tensor(o, device=local.device)] = buf[r * width:r * width + len(o)]
    return out
