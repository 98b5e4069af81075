"""Drop-in name for callers of ``breeze.cpu_backend``.

``from breeze_engine_b200 import cpu_backend as ib`` gives the same functions
(``available``, ``set_threads``, ``set_hi_prec``, ``prepack``, ``matmul``,
``free``) with the same arguments and exceptions as ``breeze/cpu_backend.py:57-242``;
the work runs on the GPU in libbreeze_ql.so (see :mod:`breeze_engine_b200.backend`).
"""
from .backend import available, free, get_hi_prec, matmul, prepack, set_hi_prec, set_threads, weight_info

__all__ = ["available", "set_threads", "set_hi_prec", "get_hi_prec", "prepack", "matmul", "free",
           "weight_info"]
