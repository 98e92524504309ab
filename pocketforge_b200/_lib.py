"""ctypes bindings of libpf_b200.so (include/pf_b200.h).

The library is the product: if it is missing the import fails loudly; there
is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpf_b200.so")

PF_OK, PF_ERR_INVALID, PF_ERR_CUDA, PF_ERR_OOM, PF_ERR_NO_DEVICE, PF_ERR_DEVICE, PF_ERR_STATE = range(7)
STATUS_NAMES = {0: "PF_OK", 1: "PF_ERR_INVALID", 2: "PF_ERR_CUDA", 3: "PF_ERR_OOM", 4: "PF_ERR_NO_DEVICE",
                5: "PF_ERR_DEVICE", 6: "PF_ERR_STATE"}


class PfError(RuntimeError):
    def __init__(self, status: int, where: str, text: str):
        super().__init__(f"{where}: {STATUS_NAMES.get(status, status)}: {text}")
        self.status = status


class ModelConfigC(C.Structure):
    _fields_ = [
        ("n_layers", C.c_int32), ("n_embd", C.c_int32), ("n_heads", C.c_int32),
        ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("n_ff", C.c_int32),
        ("n_vocab", C.c_int32), ("n_mtp_heads", C.c_int32), ("sink_size", C.c_int32),
        ("window_size", C.c_int32), ("pool_block", C.c_int32), ("max_context", C.c_int32),
        ("rope_theta", C.c_float), ("norm_eps", C.c_float), ("skip_enabled", C.c_int32),
        ("skip_threshold", C.c_float), ("qtype", C.c_int32 * 7), ("emb_qtype", C.c_int32),
    ]


class SamplingConfigC(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_uint32),
                ("greedy", C.c_int32)]


_lib = None


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is not built; run `python -m pocketforge_b200.build`")
    L = C.CDLL(LIB_PATH)
    st, vp, i32, i64, u32, f32, sz = C.c_int32, C.c_void_p, C.c_int32, C.c_int64, C.c_uint32, C.c_float, C.c_size_t

    def sig(name, res, *args):
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = list(args)

    sig("pf_last_error", C.c_char_p)
    sig("pf_device_count", i32)
    sig("pf_packed_weight_bytes", sz, i32, i32, i32)
    sig("pf_quantize_activation_rows", st, vp, vp, vp, i32, i32, vp)
    sig("pf_dequant_q4_to_int8", st, vp, vp, f32, i64, vp)
    sig("pf_dequant_q2_to_int8", st, vp, vp, f32, i64, vp)
    sig("pf_dequant_ternary_to_int8", st, vp, vp, i64, vp)
    sig("pf_matmul_int8", st, vp, vp, vp, i32, i32, i32, vp)
    sig("pf_matmul_quantized", st, vp, vp, vp, i32, i32, i32, vp, vp, vp)
    sig("pf_rmsnorm_rows", st, vp, vp, vp, i32, i32, vp)
    sig("pf_softmax_rows", st, vp, i32, i32, vp)
    sig("pf_argmax_rows", st, vp, i32, i32, vp, vp)
    sig("pf_sample_rows", st, vp, i32, i32, C.POINTER(SamplingConfigC), vp, vp, vp)
    sig("pf_pack_weights", st, vp, i32, i32, i32, vp, vp)
    sig("pf_gemm_packed", st, vp, vp, vp, vp, i32, vp, i32, i32, i32, vp)
    sig("pf_check_reciprocal", st, vp, vp)
    sig("pf_check_ordered_scan", st, vp, i32, i32, i32, vp, vp, vp)
    sig("pf_engine_create", st, C.POINTER(ModelConfigC), i32, i32, i32, C.POINTER(vp))
    sig("pf_engine_destroy", None, vp)
    sig("pf_engine_set_matrix", st, vp, i32, i32, vp, vp)
    sig("pf_engine_set_embedding", st, vp, vp, f32)
    sig("pf_engine_set_norms", st, vp, vp, vp, vp)
    sig("pf_engine_set_mtp_head", st, vp, i32, vp, vp, vp, vp, vp, vp)
    sig("pf_engine_set_sampling", st, vp, C.POINTER(SamplingConfigC))
    sig("pf_engine_set_skip_threshold", st, vp, f32)
    sig("pf_engine_prefill", st, vp, i32, vp, vp, vp)
    sig("pf_engine_step", st, vp, vp, vp)
    sig("pf_engine_run_steps", st, vp, i32)
    sig("pf_engine_set_drafts", st, vp, vp)
    sig("pf_engine_read_logits", st, vp, vp)
    sig("pf_engine_read_drafts", st, vp, vp)
    sig("pf_engine_read_pending", st, vp, vp)
    sig("pf_engine_read_positions", st, vp, vp)
    sig("pf_engine_read_hidden", st, vp, vp)
    sig("pf_engine_read_mtp_logits", st, vp, vp)
    sig("pf_engine_read_skip_counts", st, vp, C.POINTER(C.c_int64), C.POINTER(C.c_int64))
    sig("pf_engine_read_log", st, vp, vp, vp, i32)
    sig("pf_engine_read_kv", st, vp, i32, i32, i32, vp, vp, vp, vp, i32, C.POINTER(C.c_int32))
    sig("pf_engine_last_ms", st, vp, C.POINTER(C.c_float))
    sig("pf_engine_launches_per_step", st, vp, C.POINTER(C.c_int32))
    sig("pf_engine_set_kernel_timing", st, vp, C.c_int32)
    sig("pf_engine_set_attention_splits", st, vp, C.c_int32)
    sig("pf_read_device_error", st, C.POINTER(C.c_uint32), C.c_int32)
    sig("pf_engine_kernel_times", st, vp, C.POINTER(C.c_float), C.POINTER(C.c_int32))
    sig("pf_synth_matrix", st, u32, i32, i32, i32, i32, i32, vp, vp, vp)
    sig("pf_synth_mtp_matrix", st, u32, i32, i32, i32, vp, vp)
    sig("pf_engine_load_synthetic", st, vp, C.POINTER(ModelConfigC), u32, u32, i32)
    _lib = L
    return L


def check(status: int, where: str) -> None:
    if status != PF_OK:
        raise PfError(status, where, lib().pf_last_error().decode(errors="replace"))


def ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data
