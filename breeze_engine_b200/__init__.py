from . import backend, cpu_backend, linear, quant

__all__ = ["backend", "cpu_backend", "linear", "quant"]
