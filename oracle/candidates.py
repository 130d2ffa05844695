"""Two-level indexer selection oracle (numpy) -- test infrastructure, not the product.

Restates ``select_candidate_blocks`` (``src/mzoo/archs/dsv4/modeling_deepseek_v41.py:427-454``,
identical in ``archs/owlet1/indexer.py:14-41``) and the level-two selection of
``DeepseekV41Indexer.forward`` (``modeling_deepseek_v41.py:566-578``), with ties broken by
the lower block index / position (the reference leaves tie order to ``torch.topk``).
Pinned against the reference's own outputs in ``tests/golden/candidates.npz``.

- level one: pad the row to a multiple of ``block_size`` with -inf, block score = max;
  the block ``(compress_len - 1) // block_size`` (floor division) becomes +inf; keep the
  ``min(topk_blocks, n_blocks)`` best blocks whose score is > -inf.
- level two: scores outside the candidates -> -inf; the ``min(topk, T)`` best positions
  whose score is > -inf, written ascending and -1 padded.
NaN scores count as -inf (``np.fmax`` skips them).
"""

import numpy as np


def block_scores(logits: np.ndarray, compress_lens: np.ndarray, block_size: int) -> np.ndarray:
    """[rows, T] fp32, [rows] int -> [rows, n_blocks] float64 block scores with the pin."""
    rows, T = logits.shape
    nb = -(-T // block_size)
    pad = np.full((rows, nb * block_size), -np.inf, np.float64)
    x = logits.astype(np.float64)
    pad[:, :T] = np.where(np.isnan(x), -np.inf, x)
    sc = pad.reshape(rows, nb, block_size).max(axis=2)
    last = (compress_lens.astype(np.int64) - 1) // block_size  # floor division, as torch's //
    hit = np.arange(nb)[None, :] == last[:, None]
    return np.where(hit, np.inf, sc)


def _top_ascending(vals: np.ndarray, k: int) -> list:
    """Per row: indices of the k largest values > -inf (ties -> lower index), ascending."""
    out = []
    n = vals.shape[1]
    idx = np.arange(n)
    for row in vals:
        order = np.lexsort((idx, -row))[:min(k, n)]
        out.append(np.sort(order[row[order] > -np.inf]))
    return out


def candidate_blocks_ref(logits: np.ndarray, compress_lens: np.ndarray, topk_blocks: int,
                         block_size: int) -> np.ndarray:
    """int32 [rows, topk_blocks]: kept blocks ascending, -1 padded."""
    sc = block_scores(logits, compress_lens, block_size)
    out = np.full((logits.shape[0], topk_blocks), -1, np.int32)
    for r, picks in enumerate(_top_ascending(sc, topk_blocks)):
        out[r, :len(picks)] = picks
    return out


def candidate_mask_ref(logits: np.ndarray, compress_lens: np.ndarray, topk_blocks: int,
                       block_size: int) -> np.ndarray:
    """bool [rows, T]: the reference's return value."""
    rows, T = logits.shape
    nb = -(-T // block_size)
    blocks = candidate_blocks_ref(logits, compress_lens, topk_blocks, block_size)
    keep = np.zeros((rows, nb + 1), bool)
    for r in range(rows):
        b = blocks[r]
        keep[r, b[b >= 0]] = True
    return np.repeat(keep[:, :nb], block_size, axis=1)[:, :T]


def candidate_topk_ref(scores: np.ndarray, mask: np.ndarray, topk: int) -> np.ndarray:
    """int32 [rows, min(topk, T)]: best candidate positions above -inf, ascending, -1 padded."""
    rows, T = scores.shape
    width = min(topk, T)
    x = scores.astype(np.float64)
    x = np.where(mask & ~np.isnan(x), x, -np.inf)
    out = np.full((rows, width), -1, np.int32)
    for r, picks in enumerate(_top_ascending(x, width)):
        out[r, :len(picks)] = picks
    return out
