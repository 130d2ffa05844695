"""Two-level (hierarchical) indexer selection with mzoo's call signature, on sm_100a kernels.

Drop-in for ``select_candidate_blocks`` (``src/mzoo/archs/dsv4/modeling_deepseek_v41.py:427``,
identical in ``archs/owlet1/indexer.py:14``) -- level one: the ``topk_blocks`` best blocks of
``block_size`` compressed positions per query, the query's newest (partly filled) block
pinned in, returned as the reference's bool mask -- plus the compact forms the kernels use:

- ``candidate_blocks(...)`` -> int32 ``[..., topk_blocks]`` kept block indices, ascending,
  ``-1`` padded;
- ``candidate_topk(index_scores, candidates, topk)`` -> level two
  (``modeling_deepseek_v41.py:566-578``): the ``topk`` best candidate positions whose score
  is above ``-inf``, ascending, ``-1`` padded, width ``min(topk, T)``.  ``candidates`` is
  the bool mask of level one or its int32 block list.

Ties go to the lower block index / position (``torch.topk`` leaves them unspecified; the
reference's tests compare sets).  NaN scores count as ``-inf``.
"""

import torch

from . import ops
from ._lib import require_cuda


def _rows(logits: torch.Tensor, compress_lens: torch.Tensor) -> tuple:
    require_cuda(logits, compress_lens)
    lead, T = tuple(logits.shape[:-1]), logits.shape[-1]
    lg = logits.float().reshape(-1, T).contiguous()
    cl = compress_lens
    if cl.dim() == len(lead) + 1 and cl.shape[-1] == 1:  # the reference's trailing axis
        cl = cl.squeeze(-1)
    cl = cl.expand(lead).reshape(-1).clamp(-1, 2**31 - 1).to(torch.int32).contiguous()
    return lg, cl, lead, T


def candidate_blocks(logits: torch.Tensor, compress_lens: torch.Tensor, topk_blocks: int,
                     block_size: int) -> torch.Tensor:
    """int32 ``[..., topk_blocks]``: the kept blocks of ``select_candidate_blocks``, ascending."""
    lg, cl, lead, _ = _rows(logits, compress_lens)
    blocks, _ = ops.candidate_blocks(lg, cl, int(topk_blocks), int(block_size), False)
    return blocks.reshape(*lead, topk_blocks)


def select_candidate_blocks(logits: torch.Tensor, compress_lens: torch.Tensor, topk_blocks: int,
                            block_size: int) -> torch.Tensor:
    """Bool mask shaped like ``logits``: True where the position's block is a candidate."""
    lg, cl, lead, T = _rows(logits, compress_lens)
    _, mask = ops.candidate_blocks(lg, cl, int(topk_blocks), int(block_size), True)
    return mask.view(torch.bool).reshape(*lead, T)


def candidate_topk(index_scores: torch.Tensor, candidates: torch.Tensor, topk: int, *,
                   block_size: int = 8) -> torch.Tensor:
    """int32 ``[..., min(topk, T)]``: the best candidate positions (score > -inf), ascending,
    ``-1`` padded.  ``candidates``: bool mask like ``index_scores`` or an int32 block list
    ``[..., nblk]`` of ``block_size``-position blocks."""
    require_cuda(index_scores, candidates)
    lead, T = tuple(index_scores.shape[:-1]), index_scores.shape[-1]
    width = min(int(topk), T)
    if width == 0:
        return torch.full((*lead, 0), -1, dtype=torch.int32, device=index_scores.device)
    sc = index_scores.float().reshape(-1, T).contiguous()
    if candidates.dtype == torch.bool:
        assert tuple(candidates.shape) == tuple(index_scores.shape), "candidate mask must be shaped like the scores"
        mask = candidates.reshape(-1, T).contiguous().view(torch.uint8)
        out = ops.candidate_topk(sc, None, mask, 1, width)
    else:
        blocks = candidates.reshape(sc.shape[0], -1).to(torch.int32).contiguous()
        out = ops.candidate_topk(sc, blocks, None, int(block_size), width)
    return out.reshape(*lead, width)
