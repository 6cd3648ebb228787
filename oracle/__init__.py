"""CPU oracle for the grouped MoE-LoRA expert layer: TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the algorithm of the reference's routed
MoE-LoRA path (thinkube/meepsquared):

* ``routing``  -- the permutation of ``meepsquared/_moe.py:75-87`` (sort,
  histogram, cumulative offsets, gather, sentinel mask), the weighted
  un-permute of ``_moe.py:123-126`` and the tile map of
  ``meepsquared/_grouped.py:83-103``;
* ``grouped``  -- the grouped product with adapters of
  ``meepsquared/_grouped.py:420-444`` (``reference`` / ``reference_lora``) and
  the gradients of ``_LoraGroupedProduct.backward`` (``_grouped.py:385-405``),
  plus the SwiGLU gate of Transformers' ``_default_apply_gate``;
* ``quant``    -- bf16 rounding, the e4m3 format, the per-expert FP8 stacks of
  ``meepsquared/_fp8.py:122-134``, the 128x128 block FP8 of
  ``meepsquared/_vendor/axolotl/quantize.py:131-157,238-263`` and the NF4
  double quantisation that ``quantize.py:52-101`` hands to bitsandbytes 0.50.2;
* ``layer``    -- the whole routed layer, forward and backward, in float32;
* ``merge``    -- the merged save of an expert stack, ``meepsquared/_save.py:79-95``.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package, and only as
the checker or the timed CPU baseline.  The product (``meepsquared_b200``)
never imports it: without its CUDA library the product raises.

Parity pins: routing, tile map, grouped product, layer and per-expert FP8 are
pinned by golden vectors produced by the reference's own code
(``tests/golden/make_golden.py``); block FP8 by the reference's
``dequantize_fp8``/``quantize_fp8`` run with bitsandbytes stubbed out.  NF4 is
"parity unpinned": bitsandbytes is not installed, so the NF4 restatement
follows the published format (QLoRA, Dettmers et al. 2023) and its vectors are
frozen from this oracle.
"""
