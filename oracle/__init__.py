"""CPU oracle (test infrastructure only): a NumPy restatement of the reference
contextualizer, ``avey_kernels/ops.py::_reference``. Never imported by the
product package ``avey_kernel_b200``."""

from .contextualizer import ACTIVATIONS, activate, allowed_pairs, avey, avey_b, contextualize

__all__ = ['ACTIVATIONS', 'activate', 'allowed_pairs', 'avey', 'avey_b', 'contextualize']
