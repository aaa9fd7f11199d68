"""moe_engine -- B200-native batch-one decode path for the miniMoE engine.

Module layout mirrors the reference engine (``model``, ``fused_moe``,
``paged_attention``, ``checkpoint``); the kernels live in ``libmie.so`` built
from ``../csrc`` (see :mod:`moe_engine.build`) and are bound in
:mod:`moe_engine.capi`.
"""
