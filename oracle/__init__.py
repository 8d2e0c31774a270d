"""CPU oracle of the KV offload hot path - TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm may import this package, and only as the checker or the timed CPU
baseline. The product (kvoff) never imports it.
"""

from oracle.oracle import *  # noqa: F401,F403
