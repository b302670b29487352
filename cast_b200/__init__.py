"""B200-native CAST hot path: RCSA sparse attention and PAR reconstruction.

Public API:

* :func:`cast_b200.rcsa.select_quant`, :func:`cast_b200.rcsa.block_sparse_attention`,
  :func:`cast_b200.rcsa.rcsa_attention`, :func:`cast_b200.rcsa.longcat_active`
* :class:`cast_b200.par.FCPASMCorrector`
* :class:`cast_b200.select.TABASelector`
* :func:`cast_b200.components.make_cast_components` (reference-package drop-in)
* :mod:`cast_b200.distributed` (head / rollout sharding over NCCL)

Kernels live in ``libcast_b200.so`` (built by ``python -m cast_b200.build``).
"""

from . import workloads  # noqa: F401
from .rcsa import (  # noqa: F401
    Selection,
    block_sparse_attention,
    longcat_active,
    longcat_asymmetric,
    rcsa_attention,
    select_quant,
)
from .par import FCPASMCorrector  # noqa: F401
from .select import TABASelector  # noqa: F401

__version__ = "0.1.0"


def make_cast_components(**kwargs):
    from .components import make_cast_components as _mk

    return _mk(**kwargs)
