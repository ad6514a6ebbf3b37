"""CPU restatement of RESPECT's trie-verify path — TEST INFRASTRUCTURE ONLY.

This package is the checker the parity tests, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline leg compare respect_b200's CUDA path against. It is
never imported by the product (``respect_b200``), which fails loudly when its
native library is missing instead of falling back to anything here.

Each function restates, in numpy, the algorithm of the reference file:line it
cites (paths inside the soonhong99/respect project). Parity is pinned by
``tests/golden/*``: fixtures produced by running the reference's own code
(its Triton kernels under TRITON_INTERPRET=1 in fp32, its trie/acceptance
helpers, its verify_trie mask builder, HF eager) in the build container with
``tests/golden/make_golden.py``; ``tests/test_oracle_golden.py`` checks this
package against them.
"""
