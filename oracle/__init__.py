"""CPU oracle for the Sticky-KV decode hot path -- TEST INFRASTRUCTURE ONLY.

This package is a numpy restatement of the reference algorithm
(shaswata965-coder/Qevict, ``src/models/kv_cache`` and ``src/models/attention``).
Every function cites the reference file:line it follows.

It exists to check the CUDA path, never to serve it: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it.
The product package ``qevict_b200`` never imports anything from here and fails
loudly when its CUDA library is missing.

Parity pin: the oracle is checked against golden vectors produced by running
the reference itself (``tests/golden/make_golden.py`` imports the reference's
own Python modules and records their outputs into ``tests/golden/*.npz``;
``tests/test_oracle_golden.py`` replays them through this package).
"""

from .numerics import rnd, f32, DTYPES  # noqa: F401
