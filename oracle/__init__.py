"""CPU oracle of D2-SD's tree-verification hot path.

TEST INFRASTRUCTURE ONLY. This package restates, on the CPU, the reference
algorithms the CUDA kernels replace. Only ``tests/``, ``__graft_entry__.smoke()``
and the CPU-baseline leg of ``bench.py`` may import it, and only as the checker
or the timed CPU baseline -- never as part of the product path, which fails
loudly when its CUDA library is missing.

Modules
-------
attention  FlashInfer-convention attention (base-2 LSE), state merge, the
           two-level cascade of generation/verification.py:127-176 and
           model/cascade_graph.py:52-60, and the torch.sdpa masked path.
accept     greedy acceptance, generation/d3_generator.py:204-225 and
           generation/dflash_generator.py:110-125.
commit     accepted-branch KV commit, generation/d3_generator.py:227-232,
           on a contiguous cache and on a paged cache.

Pinning: tests/golden/make_golden.py runs the reference's own code in the
container that holds it (the acceptance and commit blocks executed from the
reference source, the reference's cascade_verify_forward against its
plain_verify_forward) and stores the results as fixtures that
tests/test_oracle_golden.py checks this oracle against.
"""
