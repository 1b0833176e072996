"""CPU oracle for the int4/int8 weight-only linear path and the fused attention.

TEST INFRASTRUCTURE ONLY. Nothing in the product package imports this
package; only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use it, and only
as the checker or as the timed CPU stand-in for the reference's own CPU torch
path. The GPU path fails loudly when its CUDA library is missing; it never
falls back to anything here.
"""
from .oracle import *  # noqa: F401,F403
from .attention import *  # noqa: F401,F403
