"""Rebind the reference package's INT8 hot path to ksdraft_b200.

    import ksdraft_b200.install as kb
    kb.install()            # before anything imports ksdraft.kernels
    import ksdraft          # KSDraftModel, the staged trainer, export: unchanged

Whole modules are replaced where this package mirrors every public name of
the reference module (ksdraft/kernels/{quant,gemm,linear,ks3_int8,
ks3_triton,rosa_credit_gpu}.py): their entries in `sys.modules` point at the
mirrors, so the reference's own `from .quant import ...` statements (and
RosaMixer's `from ..kernels.rosa_credit_gpu import HardRosaGPU`) bind the B200
code.
Where the reference module holds more than the hot path, single functions
are patched instead:
  ksdraft/model/rosa.py:40      _match_payload_sign (RosaMixer.forward looks
                                it up at call time, rosa.py:161)
  ksdraft/train/stages.py:27    quantize_last_dim_dithered
"""

from __future__ import annotations

import importlib
import importlib.util
import sys

KERNEL_MODULES = ("quant", "gemm", "linear", "ks3_int8", "ks3_triton", "rosa_credit_gpu")
PATCHED_FUNCTIONS = (
    ("model.rosa", "_match_payload_sign", "ksdraft_b200.model.rosa"),
    ("train.stages", "quantize_last_dim_dithered", "ksdraft_b200.train.stages"),
)


def install(package: str = "ksdraft") -> dict[str, str]:
    """Point `package`'s hot-path modules and functions at ksdraft_b200.

    Must run before `package.kernels` is imported (a module that already bound
    the reference functions with `from ... import` would keep them): raises
    RuntimeError otherwise.  Returns {reference name: replacement name}."""
    done: dict[str, str] = {}
    for name in KERNEL_MODULES:
        ref = f"{package}.kernels.{name}"
        if ref in sys.modules and not getattr(sys.modules[ref], "__ksdraft_b200__", False):
            raise RuntimeError(f"{ref} was imported before ksdraft_b200.install.install()")
    for name in KERNEL_MODULES:
        mine = importlib.import_module(f"ksdraft_b200.kernels.{name}")
        mine.__ksdraft_b200__ = True
        sys.modules[f"{package}.kernels.{name}"] = mine
        done[f"{package}.kernels.{name}"] = mine.__name__
    parent = importlib.import_module(f"{package}.kernels")
    for name in KERNEL_MODULES:     # attribute access (ksdraft.kernels.gemm) too
        setattr(parent, name, sys.modules[f"{package}.kernels.{name}"])
    for sub, func, mine_name in PATCHED_FUNCTIONS:
        if importlib.util.find_spec(f"{package}.{sub}") is None:
            continue   # a reference version without this module
        ref_mod = importlib.import_module(f"{package}.{sub}")
        mine = importlib.import_module(mine_name)
        setattr(ref_mod, func, getattr(mine, func))
        done[f"{package}.{sub}.{func}"] = f"{mine_name}.{func}"
    return done
