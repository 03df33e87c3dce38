"""CPU oracle for the quantized decode path (test infrastructure only).

Nothing in the shipped package imports this directory. Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline legs of ``bench.py`` use it,
always as the checker or the timed CPU reference, never as the product path.
"""

from .axb_oracle import *  # noqa: F401,F403
