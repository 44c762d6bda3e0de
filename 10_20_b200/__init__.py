"""v1x: B200-native (sm_100a) query-side selection path of the SGLang V1
sparse-attention index backend.

Drop-in modules mirroring the reference's operator surfaces:
  query_fused     module().route / .topk           (v1_deepseek/query_fused.py)
  kernels         Triton-style page-lifecycle and query ops (v1_deepseek/kernels.py)
  fused_grouping  _sort                            (v1_native/fused_grouping.py)
  gather          _gather_slots, GatherWorkspace   (v1_native/kernels.py)
  scoring         fp8_paged_mqa_logits             (DeepGEMM contract)
and the composed step (`pipeline.SelectionStep`) plus seeded synthetic
workloads (`synth`).  All compute runs in libv1x.so; there is no CPU path.

The package directory name is not a Python identifier: import it with
``importlib.import_module("10_20_b200")``.
"""
from . import _lib  # noqa: F401

__version__ = "0.1.0"


def library_path() -> str:
    return str(_lib.LIB_PATH)


def load() -> None:
    """Load libv1x.so now (raises if it is missing)."""
    _lib.lib()
