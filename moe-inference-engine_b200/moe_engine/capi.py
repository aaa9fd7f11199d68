"""ctypes binding of ``libmie.so`` (the C ABI declared in ``include/mie.h``).

The structures below mirror the C structs field for field.  Device pointers
are passed as integers (``tensor.data_ptr()``), streams as the raw
``cudaStream_t`` of the current torch stream.  There is no CPU fallback: when
the library is missing every entry point raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_native", "libmie.so")

MIE_OK, MIE_ERR_INVALID, MIE_ERR_UNSUPPORTED, MIE_ERR_CUDA, MIE_ERR_TIMEOUT, MIE_ERR_RANGE, MIE_ERR_SCRATCH_LIMIT = range(7)
MIE_STEP_AUTO, MIE_STEP_FLAT, MIE_STEP_CLUSTER = range(3)
MIE_F32, MIE_BF16 = 0, 1
MIE_NORM_NONE, MIE_NORM_RMS, MIE_NORM_LAYER = 0, 1, 2
MIE_ACT_GELU, MIE_ACT_SWIGLU = 0, 1

_i, _f, _p, _i64 = ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_int64


class MoeArgs(ctypes.Structure):
    _fields_ = [
        ("dtype", _i), ("x_dtype", _i), ("out_dtype", _i), ("hidden_dim", _i),
        ("expert_hidden_dim", _i), ("num_experts", _i), ("top_k", _i), ("act", _i),
        ("norm", _i), ("eps", _f), ("x", _p), ("norm_w", _p), ("norm_b", _p),
        ("router_w", _p), ("w1", _p), ("b1", _p), ("w3", _p), ("w2", _p), ("b2", _p),
        ("router_logits", _p), ("expert_ids", _p), ("route_weights", _p), ("hidden", _p),
        ("out", _p), ("residual", _i), ("sync", _p), ("status", _p), ("skip", _p),
        ("grid", _i), ("expert_base", _i), ("expert_count", _i),
        ("expert_bits", _i), ("group_size", _i), ("w1_scale", _p), ("w3_scale", _p), ("w2_scale", _p),
        ("peer_rank", _i), ("peer_world", _i), ("peer_seq", _p), ("peer_bufs", _p * 8),
        ("peer_wait_limit_ns", _i64),
    ]


class AttnArgs(ctypes.Structure):
    _fields_ = [
        ("kv_dtype", _i), ("q_dtype", _i), ("out_dtype", _i), ("num_heads", _i), ("head_dim", _i),
        ("q", _p), ("k", _p), ("v", _p), ("block_table", _p), ("num_blocks", _i),
        ("block_size", _i), ("stride_block", _i64), ("stride_head", _i64), ("stride_tok", _i64),
        ("ctx_len", _i), ("ctx_dev", _p), ("ctx_dev_offset", _i), ("max_ctx", _i), ("scale", _f),
        ("out", _p), ("partials", _p), ("counters", _p), ("splits", _i), ("max_splits", _i),
        ("new_token_last", _i), ("status", _p), ("skip", _p), ("defer_merge", _i),
    ]


class QkvArgs(ctypes.Structure):
    _fields_ = [
        ("dtype", _i), ("kv_dtype", _i), ("hidden_dim", _i), ("num_heads", _i), ("head_dim", _i),
        ("norm", _i), ("eps", _f), ("norm_w", _p), ("norm_b", _p), ("x", _p), ("x_add", _p),
        ("embedding", _p), ("pos_embedding", _p), ("token", _p), ("vocab", _i), ("w", _p),
        ("b", _p), ("rope_cos", _p), ("rope_sin", _p), ("pos", _p), ("max_pos", _i),
        ("q_out", _p), ("k_cache", _p), ("v_cache", _p), ("block_table", _p), ("num_blocks", _i),
        ("block_size", _i), ("stride_block", _i64), ("stride_head", _i64), ("stride_tok", _i64),
        ("status", _p), ("skip", _p), ("grid", _i),
    ]


class ProjArgs(ctypes.Structure):
    _fields_ = [
        ("dtype", _i), ("rows", _i), ("cols", _i), ("w", _p), ("b", _p), ("in_", _p),
        ("out", _p), ("add", _p), ("accumulate", _i), ("status", _p), ("skip", _p), ("grid", _i),
        ("attn_partials", _p), ("attn_heads", _i), ("attn_head_dim", _i), ("attn_splits", _i),
        ("attn_max_splits", _i),
    ]


class LmHeadArgs(ctypes.Structure):
    _fields_ = [
        ("dtype", _i), ("vocab", _i), ("hidden_dim", _i), ("norm", _i), ("eps", _f),
        ("norm_w", _p), ("norm_b", _p), ("x", _p), ("x_add", _p), ("w", _p), ("b", _p),
        ("logits", _p), ("partial_val", _p), ("partial_idx", _p), ("counter", _p),
        ("token_out", _p), ("pos", _p), ("tokens_log", _p), ("log_count", _p),
        ("log_capacity", _i), ("done", _p), ("eos_id", _i), ("status", _p), ("skip", _p),
        ("grid", _i),
    ]


class LayerDesc(ctypes.Structure):
    _fields_ = [
        ("attn_norm_w", _p), ("attn_norm_b", _p), ("qkv_w", _p), ("qkv_b", _p), ("out_w", _p),
        ("out_b", _p), ("moe_norm_w", _p), ("moe_norm_b", _p), ("router_w", _p), ("w1", _p),
        ("b1", _p), ("w3", _p), ("w2", _p), ("b2", _p), ("k_cache", _p), ("v_cache", _p),
        ("w1_scale", _p), ("w3_scale", _p), ("w2_scale", _p),
    ]


class StepDesc(ctypes.Structure):
    _fields_ = [
        ("dtype", _i), ("kv_dtype", _i), ("num_layers", _i), ("hidden_dim", _i), ("num_heads", _i),
        ("head_dim", _i), ("num_experts", _i), ("top_k", _i), ("expert_hidden_dim", _i),
        ("vocab", _i), ("norm", _i), ("act", _i), ("eps", _f), ("attn_scale", _f), ("max_pos", _i),
        ("layers", _p), ("embedding", _p), ("pos_embedding", _p), ("final_norm_w", _p),
        ("final_norm_b", _p), ("lm_bias", _p), ("rope_cos", _p), ("rope_sin", _p),
        ("block_table", _p), ("num_blocks", _i), ("block_size", _i), ("kv_stride_block", _i64),
        ("kv_stride_head", _i64), ("kv_stride_tok", _i64), ("token", _p), ("pos", _p),
        ("done", _p), ("eos_id", _i), ("tokens_log", _p), ("log_count", _p), ("log_capacity", _i),
        ("x", _p), ("q", _p), ("attn_out", _p), ("moe_hidden", _p), ("moe_partial", _p),
        ("expert_base", _i), ("expert_count", _i), ("attn_partials", _p), ("attn_counters", _p),
        ("moe_sync", _p), ("lm_partial_val", _p), ("lm_partial_idx", _p), ("lm_counter", _p),
        ("logits", _p), ("status", _p), ("attn_splits", _i), ("max_splits", _i), ("lm_grid", _i),
        ("use_pdl", _i), ("step_scratch", _p), ("step_scratch_bytes", _i64), ("sample_temperature", _f),
        ("sample_top_k", _i), ("sample_seed", _p), ("step_limit", _p), ("wait_limit_ns", _i64),
        ("start_gate", _p), ("step_kernel", _i), ("moe_peer", _p), ("expert_bits", _i), ("group_size", _i),
    ]


GEMM_F32, GEMM_BF16, GEMM_RESID, GEMM_SWIGLU, GEMM_GELU = 0, 1, 2, 3, 4


class GemmArgs(ctypes.Structure):
    _fields_ = [
        ("a", _p), ("lda", _i64), ("b", _p), ("b2", _p), ("ldb", _i64), ("b_rows", _i64), ("c", _p),
        ("ldc", _i64), ("resid", _p), ("ldr", _i64), ("counts", _p), ("M", _i), ("N", _i), ("K", _i),
        ("epilogue", _i), ("groups", _i), ("a_group_rows", _i), ("b_group_rows", _i),
        ("c_group_rows", _i), ("status", _p), ("bias", _p), ("bias_group_stride", _i64),
    ]


class PrefillNormArgs(ctypes.Structure):
    _fields_ = [
        ("tokens", _i), ("hidden_dim", _i), ("norm", _i), ("eps", _f), ("ids", _p), ("embedding", _p),
        ("pos_embedding", _p), ("pos0", _i), ("x", _p), ("w", _p), ("b", _p), ("out", _p),
    ]


class PrefillAttnArgs(ctypes.Structure):
    _fields_ = [
        ("tokens", _i), ("num_heads", _i), ("head_dim", _i), ("scale", _f), ("q", _p), ("k", _p), ("v", _p),
        ("out", _p), ("ld_out", _i64), ("status", _p),
    ]


MIE_PEER_MAX_RANKS = 8


class PeerReduceArgs(ctypes.Structure):
    _fields_ = [
        ("n", _i), ("rank", _i), ("world", _i), ("in_", _p), ("out", _p), ("bufs", _p * MIE_PEER_MAX_RANKS),
        ("seq", _p), ("status", _p), ("wait_limit_ns", _i64),
    ]


class PrefillRopeArgs(ctypes.Structure):
    _fields_ = [
        ("tokens", _i), ("num_heads", _i), ("head_dim", _i), ("pos0", _i), ("qkv", _p), ("rope_cos", _p),
        ("rope_sin", _p), ("q_out", _p), ("k_out", _p), ("v_out", _p), ("k_cache", _p), ("v_cache", _p),
        ("block_table", _p), ("block_size", _i), ("kv_stride_block", _i64), ("kv_stride_head", _i64),
        ("kv_stride_tok", _i64),
    ]


class PrefillRouteArgs(ctypes.Structure):
    _fields_ = [
        ("tokens", _i), ("hidden_dim", _i), ("num_experts", _i), ("group_rows", _i), ("x", _p),
        ("x_res", _p), ("norm", _i), ("eps", _f), ("norm_w", _p), ("norm_b", _p),
        ("router_w", _p), ("logits", _p), ("counts", _p), ("weights", _p), ("ids_out", _p),
        ("rows_out", _p), ("gathered", _p),
    ]


class PrefillCombineArgs(ctypes.Structure):
    _fields_ = [
        ("tokens", _i), ("hidden_dim", _i), ("x", _p), ("y", _p), ("ldy", _i64), ("weights", _p),
        ("rows", _p),
    ]


# Every symbol include/mie.h declares, with its ctypes argument types.
SYMBOLS = {
    "mie_version": ([], ctypes.c_int),
    "mie_init": ([_i], ctypes.c_int),
    "mie_status_string": ([_i], ctypes.c_char_p),
    "mie_last_cuda_error": ([], ctypes.c_char_p),
    "mie_num_sms": ([_i], ctypes.c_int),
    "mie_moe_route": ([ctypes.POINTER(MoeArgs), _p], ctypes.c_int),
    "mie_moe_decode": ([ctypes.POINTER(MoeArgs), _p], ctypes.c_int),
    "mie_attn_decode": ([ctypes.POINTER(AttnArgs), _p], ctypes.c_int),
    "mie_attn_decode_fixed_scratch": ([ctypes.POINTER(AttnArgs), _p], ctypes.c_int),
    "mie_qkv_rope_store": ([ctypes.POINTER(QkvArgs), _p], ctypes.c_int),
    "mie_proj_residual": ([ctypes.POINTER(ProjArgs), _p], ctypes.c_int),
    "mie_lmhead_argmax": ([ctypes.POINTER(LmHeadArgs), _p], ctypes.c_int),
    "mie_decode_step": ([ctypes.POINTER(StepDesc), _p], ctypes.c_int),
    "mie_decode_layer": ([ctypes.POINTER(StepDesc), _i, _p], ctypes.c_int),
    "mie_decode_head": ([ctypes.POINTER(StepDesc), _p], ctypes.c_int),
    "mie_step_scratch_bytes": ([ctypes.POINTER(StepDesc)], ctypes.c_int64),
    "mie_step_kernel_of": ([ctypes.POINTER(StepDesc)], ctypes.c_int),
    "mie_prefill_attention": ([ctypes.POINTER(PrefillAttnArgs), _p], ctypes.c_int),
    "mie_peer_buffer_bytes": ([ctypes.c_int, ctypes.c_int], ctypes.c_int64),
    "mie_peer_reduce": ([ctypes.POINTER(PeerReduceArgs), _p], ctypes.c_int),
    "mie_peer_alloc": ([ctypes.c_int64, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "mie_peer_free": ([_p], ctypes.c_int),
    "mie_peer_handle": ([_p, _p], ctypes.c_int),
    "mie_peer_open": ([_p, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "mie_peer_close": ([_p], ctypes.c_int),
    "mie_gemm": ([ctypes.POINTER(GemmArgs), _p], ctypes.c_int),
    "mie_prefill_norm": ([ctypes.POINTER(PrefillNormArgs), _p], ctypes.c_int),
    "mie_prefill_rope_kv": ([ctypes.POINTER(PrefillRopeArgs), _p], ctypes.c_int),
    "mie_prefill_route": ([ctypes.POINTER(PrefillRouteArgs), _p], ctypes.c_int),
    "mie_prefill_combine": ([ctypes.POINTER(PrefillCombineArgs), _p], ctypes.c_int),
}

_lib = None
_lock = threading.Lock()
_initialised_devices: set = set()


class KernelError(RuntimeError):
    """A libmie entry point returned a failure status."""

    def __init__(self, code: int, what: str):
        self.code = code
        detail = ""
        if code == MIE_ERR_CUDA and _lib is not None:
            detail = " [" + _lib.mie_last_cuda_error().decode() + "]"
        super().__init__(f"{what}: {status_string(code)} (status {code}){detail}")


def library_available() -> bool:
    return os.path.exists(LIB_PATH)


def load() -> ctypes.CDLL:
    """Load libmie.so (raises if it was not built)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"libmie.so not found at {LIB_PATH}; build it with "
                    "`python -c 'import __graft_entry__ as g; g.build()'` or moe_engine.build.build()"
                )
            lib = ctypes.CDLL(LIB_PATH)
            for name, (argtypes, restype) in SYMBOLS.items():
                fn = getattr(lib, name)
                fn.argtypes = argtypes
                fn.restype = restype
            _lib = lib
    return _lib


def status_string(code: int) -> str:
    try:
        return load().mie_status_string(int(code)).decode()
    except Exception:  # library missing: describe the code locally
        return {0: "ok", 1: "invalid argument", 2: "unsupported", 3: "CUDA error", 4: "timeout", 5: "range"}.get(
            int(code), "unknown status"
        )


def ensure_init(device: torch.device) -> ctypes.CDLL:
    """Load the library and set kernel attributes once per device.

    Must run before any CUDA-graph capture that launches these kernels.
    """
    lib = load()
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _initialised_devices:
        with torch.cuda.device(idx):
            rc = lib.mie_init(idx)
        if rc != MIE_OK:
            raise KernelError(rc, "mie_init")
        _initialised_devices.add(idx)
    return lib


def check(rc: int, what: str) -> None:
    if rc == MIE_OK:
        return
    if rc in (MIE_ERR_INVALID,):
        raise ValueError(f"{what}: {status_string(rc)} (status {rc})")
    raise KernelError(rc, what)


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return MIE_F32
    if dtype == torch.bfloat16:
        return MIE_BF16
    raise RuntimeError(f"the sm_100a kernels support float32 and bfloat16, not {dtype}")


def stream_handle(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t) -> int | None:
    """Device pointer of a tensor (None -> NULL)."""
    return None if t is None else t.data_ptr()
