"""CPU oracle for the mzoo attention hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy (float32 / float64 on the host), the arithmetic of
pmonad/mzoo's pure-PyTorch reference for the path the CUDA library replaces:

- ``oracle.quant``     fp8 / fp4 fake-quant rules (``src/mzoo/archs/owlet1/quant.py``)
                       plus the OCP-MXFP4 and FP8-per-tile-absmax rules;
- ``oracle.attention`` window / sparse shared-latent attention, forward and backward
                       (``src/mzoo/layers/attn/golden_ref.py``);
- ``oracle.indexer``   lightning-indexer scores and top-k
                       (``golden_ref.py:213-243``, ``indexer/fwd.py``, ``indexer/bwd.py``);
- ``oracle.mla``       576/512 latent sparse prefill and paged decode over FP8 rows;
- ``oracle.candidates`` two-level block selection (``select_candidate_blocks``,
                       ``archs/dsv4/modeling_deepseek_v41.py:427-454``);
- ``oracle.compressor`` the compressor's pool / RMSNorm / RoPE / cache-entry step
                       (``DeepseekV41Compressor``);
- ``oracle.norm_rope`` fused RMSNorm + RoPE of q / kv, forward and backward
                       (``src/mzoo/layers/attn/norm_rope.py``);
- ``oracle.kvcache``   fp8 window / fp4 main cache codes and scales (the model's
                       ``_fake_quant_fp8_block`` / ``_fake_quant_fp4_block`` as storage);
- ``oracle.torch_ref`` the same reference arithmetic in torch float32 (the CPU path the
                       benchmark's reference arm times on the host cores).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import it, and only as the checker.  The product path (``mzoo_b200``) never imports
anything from here and has no CPU fallback.

Pinning: ``tests/golden/`` holds input/output vectors produced by importing the
reference itself (``tests/golden/make_golden.py``); the CPU tests of ``tests/test_quant.py``,
``test_attn.py``, ``test_indexer.py``, ``test_sparse_mla.py``, ``test_candidates.py``,
``test_compressor.py``, ``test_norm_rope.py``, ``test_kvcache.py`` and ``test_torch_ref.py``
check this oracle against them bit-for-bit (quant, cache codes, row packing, top-k sets) or
to fp32 rounding (attention, scores).
"""
