"""CPU oracle for the FP8 MoE hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its
``cpu_baseline`` leg and ``--impl reference``) may import this package, and
only as the checker or the timed CPU baseline.  The product package
(``glm53_flash_mlx_b200``) never imports it and has no CPU fallback.

The arithmetic lives in ``oracle.c`` (a C restatement of the reference Metal
kernels, each function citing the reference file:line it follows);
``reference.py`` composes those primitives the way the reference's Python
modules do.  Parity pins are listed in the header of ``oracle.c``.
"""

from .reference import *  # noqa: F401,F403
