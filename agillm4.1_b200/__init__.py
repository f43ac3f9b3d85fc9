"""B200 (sm_100a) MoE block forward for AGILLM4.1.

Import as ``agillm41_b200`` (the repository-root alias for this directory).

* :class:`MoEFFN` - drop-in for the reference ``MoEFFN`` (agillm41.py:4323-4460)
* :func:`install` - rebind the reference runtime's ``MoEFFN`` to the B200 forward
* :func:`collect_moe_aux` - the reference's ``_collect_moe_aux`` on the fused aux-loss kernels
* :mod:`.codec`   - the reference's tensor-state codec decoded (and applied) on the GPU
* :mod:`.ops`     - one Python entry point per kernel stage, plus the fused forward
* :mod:`.torch_ops` - the same stages registered as torch operators (``torch.ops.agillm_moe``)
* :mod:`._lib`    - the ctypes binding of ``lib/libagillm_moe.so``
"""
from ._lib import LIB_PATH, MoEKernelError, load  # noqa: F401
from .moe import MoEFFN, collect_moe_aux, install, uninstall  # noqa: F401
from . import codec, ops, torch_ops  # noqa: F401

__all__ = ["MoEFFN", "collect_moe_aux", "install", "uninstall", "codec", "ops", "torch_ops", "load", "LIB_PATH", "MoEKernelError"]
