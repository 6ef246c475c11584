"""CPU oracle of the latent-KV decode path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline arm may import this package, and only
as the checker or the timed CPU baseline. The product (``belt_b200``) never imports it: a missing CUDA library
raises instead of falling back to anything here.

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here against golden vectors that
``tests/golden/make_golden.py`` produced by running the reference's own code (its torch functions, and its Triton
kernels under the Triton interpreter) in the build container.
"""

from .latent_ref import *  # noqa: F401,F403
