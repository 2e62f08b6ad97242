"""CPU oracle for the Verace V1 SSSD + CHAM sequence-mixing path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this module.
It is used by ``tests/`` (as the parity checker), by ``__graft_entry__.smoke()``
(to check one small CUDA invocation) and by ``bench.py``'s CPU-baseline /
reference arm (timed as the reference's CPU algorithm).  It is never the thing
measured for the GPU numbers and never a fallback for the CUDA path.
"""

from .verace_oracle import *  # noqa: F401,F403
