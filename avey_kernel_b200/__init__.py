"""B200-native (sm_100a) Avey and Avey-B contextualizer forward.

Drop-in for the reference package ``avey_kernels``: the same ``avey`` and
``avey_b`` entry points, backed by hand-written CUDA behind a C ABI
(``include/avey_b200.h``, ``lib/libavey_b200.so``).
"""

from .ops import avey, avey_b

__all__ = ['avey', 'avey_b']
