"""CPU oracle for the attention forward path -- TEST INFRASTRUCTURE ONLY.

Nothing in the product (the ``gfx906_b200`` package) imports this package. It
is used by ``tests/`` as the checker, by ``__graft_entry__.smoke()`` to check
one small GPU call, and by ``bench.py``'s CPU-baseline leg (and its
``--impl reference`` arm) as the reference's CPU path that is timed beside the
GPU kernel.

Contents:

* ``sdpa_math``: the reference's own oracle -- torch
  ``scaled_dot_product_attention`` under the MATH backend -- evaluated in fp32
  on the fp16 inputs, chunked over query rows for long sequences (the
  reference's slice trick). Reference call sites: ``test.py:12``,
  ``test_variants.py:54-56``, ``test_d512.py:13-14``; MATH is the only SDPA
  backend on gfx906 (``deploy/gfx906_attention.py:17-18``).
* ``online_softmax``: a numpy restatement of the reference kernel's tiled
  online softmax (``attn_kernel.hip:357, 452-462, 491-497``), with the key-tile
  size and the lazy-rescale threshold as parameters so that it also models the
  sm_100a kernel's tiling. Pinned against golden vectors produced by the
  reference's own numpy model (``model_check.py:103-153``, see
  ``tests/golden/make_golden.py``).
"""
