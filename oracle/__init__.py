"""ctypes bindings of the test oracle.

TEST INFRASTRUCTURE ONLY: the CPU restatement (liboracle.so, from
pf_oracle.cpp) and, where it was built, the reference's own functions
(_ref/libpfref.so).  Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline legs may import this package; pocketforge_b200 never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
# the reference checkout: PF_REFERENCE_DIR, else a "reference" directory beside the repository
REF_CHECKOUT = os.environ.get("PF_REFERENCE_DIR",
                              os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
u32, i32, f32, u64, vp = C.c_uint32, C.c_int32, C.c_float, C.c_uint64, C.c_void_p


class PfModelConfig(C.Structure):
    """pf_model_config of include/pf_b200.h."""

    _fields_ = [
        ("n_layers", C.c_int32), ("n_embd", C.c_int32), ("n_heads", C.c_int32),
        ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("n_ff", C.c_int32),
        ("n_vocab", C.c_int32), ("n_mtp_heads", C.c_int32), ("sink_size", C.c_int32),
        ("window_size", C.c_int32), ("pool_block", C.c_int32), ("max_context", C.c_int32),
        ("rope_theta", C.c_float), ("norm_eps", C.c_float), ("skip_enabled", C.c_int32),
        ("skip_threshold", C.c_float), ("qtype", C.c_int32 * 7), ("emb_qtype", C.c_int32),
    ]


class PfSamplingConfig(C.Structure):
    """pf_sampling_config of include/pf_b200.h (SamplingConfig)."""

    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_uint32),
                ("greedy", C.c_int32)]


def build(quiet: bool = True) -> None:
    """Builds liboracle.so and, when the reference checkout exists,
    _ref/libpfref.so and (once pocketforge_b200's library is built) the
    reference's unit tests against the forge:: headers, _ref/forge_tests/."""
    targets = ["all"]
    if os.path.exists(os.path.join(os.path.dirname(HERE), "pocketforge_b200", "libforge_b200.so")):
        targets.append("forge_tests")
    out = subprocess.run(["make", "-C", HERE, f"REF={REF_CHECKOUT}", "-j8", *targets],
                         capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)


def _sig(lib, name, res, *args):
    fn = getattr(lib, name)
    fn.restype = res
    fn.argtypes = list(args)
    return fn


_lib = None
_ref = None


def lib():
    """The CPU restatement (built on first use)."""
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path) or os.path.getmtime(path) < os.path.getmtime(
                os.path.join(HERE, "pf_oracle.cpp")):
            build()
        L = C.CDLL(path)
        _sig(L, "po_quantize_activation_row", None, _f32p, _i8p, _f32p, u32)
        _sig(L, "po_kv_quantize_row", None, _f32p, _i8p, _f32p, u32)
        _sig(L, "po_dequant_q4_to_int8", None, _u8p, _i8p, u64)
        _sig(L, "po_dequant_q2_to_int8", None, _u8p, _i8p, u64)
        _sig(L, "po_dequant_ternary_to_int8", None, _u8p, _i8p, u64)
        _sig(L, "po_matmul_int8", None, _i8p, _i8p, _i32p, u32, u32, u32)
        _sig(L, "po_matmul_quantized", None, _f32p, _i8p, _f32p, u32, u32, u32, _f32p, vp)
        _sig(L, "po_rmsnorm", None, _f32p, _f32p, _f32p, u32, f32, C.c_int)
        _sig(L, "po_softmax", None, _f32p, u32)
        _sig(L, "po_swiglu_engine", f32, f32, f32)
        _sig(L, "po_silu_mtp", f32, f32)
        _sig(L, "po_argmax", i32, _f32p, u32)
        _sig(L, "po_sample", i32, _f32p, u32, C.POINTER(PfSamplingConfig), f32)
        _sig(L, "po_sample_top_p", i32, _f32p, u32, f32, f32, f32)
        _sig(L, "po_sample_top_k", i32, _f32p, u32, u32, f32, f32)
        _sig(L, "po_uniforms", None, u32, u32, _f32p)
        _sig(L, "po_rope_table", None, f32, u32, u32, _f32p, _f32p)
        _sig(L, "po_quantize_matrix", u64, _f32p, u32, u32, C.c_int, vp)
        _sig(L, "po_loader_decode", None, _u8p, u64, u32, u32, C.c_int, _i8p, _f32p, _f32p)
        _sig(L, "po_synth_matrix", None, u32, u32, u32, u32, u32, C.c_int, _i8p, _f32p, _f32p)
        _sig(L, "po_synth_normals", None, u32, u32, u32, u64, _f32p)
        _sig(L, "po_mtp_quantize_q4", None, _f32p, _u8p, _f32p, u32, u32)
        _sig(L, "po_synth_mtp_matrix", None, u32, u32, u32, u32, _u8p, _f32p)
        _sig(L, "po_mtp_forward", None, u32, u32, _u8p, _f32p, _f32p, _f32p, u32, _f32p, vp)
        _sig(L, "po_kv_create", vp, u32, u32, u32, u32, u32, u32, u32)
        _sig(L, "po_kv_destroy", None, vp)
        _sig(L, "po_kv_store", None, vp, u32, u32, u32, _f32p, _f32p)
        _sig(L, "po_kv_scores", u32, vp, u32, u32, _f32p, _f32p)
        _sig(L, "po_kv_weighted_sum", None, vp, u32, u32, _f32p, _f32p, u32)
        _sig(L, "po_kv_count", u32, vp, u32, u32)
        _sig(L, "po_kv_size", u32, vp)
        _sig(L, "po_kv_dump", u32, vp, u32, u32, _i8p, _f32p, _i8p, _f32p, u32)
        _sig(L, "po_kv_acc", u32, vp, u32, u32, _f64p, _f64p)
        _sig(L, "po_skip_create", vp, u32, u32, f32)
        _sig(L, "po_skip_destroy", None, vp)
        _sig(L, "po_skip_should_skip", C.c_int, vp, u32, _f32p, C.c_int)
        _sig(L, "po_skip_set_threshold", None, vp, f32)
        _sig(L, "po_skip_delta", f32, _f32p, _f32p, u32, C.c_int)
        _sig(L, "po_engine_create", vp, C.POINTER(PfModelConfig))
        _sig(L, "po_engine_destroy", None, vp)
        _sig(L, "po_engine_set_order", None, vp, C.c_int)
        _sig(L, "po_engine_set_sampling", None, vp, C.POINTER(PfSamplingConfig))
        _sig(L, "po_engine_set_skip_threshold", None, vp, f32)
        _sig(L, "po_engine_set_matrix", None, vp, u32, u32, _i8p, _f32p)
        _sig(L, "po_engine_set_embedding", None, vp, _i8p, f32)
        _sig(L, "po_engine_set_norms", None, vp, vp, vp, vp)
        _sig(L, "po_engine_set_mtp_head", None, vp, u32, _u8p, _f32p, _u8p, _f32p, _u8p, _f32p)
        _sig(L, "po_engine_prefill", None, vp, i32, _i32p, _i64p, vp)
        _sig(L, "po_engine_step", None, vp, vp, vp)
        _sig(L, "po_engine_read_logits", None, vp, _f32p)
        _sig(L, "po_engine_read_drafts", None, vp, _i32p)
        _sig(L, "po_engine_set_drafts", None, vp, _i32p)
        _sig(L, "po_engine_read_pending", None, vp, _i32p)
        _sig(L, "po_engine_read_positions", None, vp, _i32p)
        _sig(L, "po_engine_read_hidden", None, vp, _f32p)
        _sig(L, "po_engine_read_mtp_logits", None, vp, _f32p)
        _sig(L, "po_engine_read_skip_counts", None, vp, C.POINTER(C.c_int64), C.POINTER(C.c_int64))
        _sig(L, "po_engine_skip_margin", C.c_float, vp)
        _sig(L, "po_engine_read_kv", u32, vp, i32, u32, u32, _i8p, _f32p, _i8p, _f32p, u32)
        _sig(L, "po_engine_probe_row", None, vp, i32, i32, _f32p, _f32p)
        _sig(L, "po_engine_load_synthetic", None, vp, u32, u32, C.c_int)
        _sig(L, "po_engine_set_threads", None, vp, C.c_int)
        _sig(L, "po_engine_set_prefill_threads", None, vp, C.c_int)
        _lib = L
    return _lib


def ref_available() -> bool:
    """True when _ref/libpfref.so exists or can be built from the checkout."""
    path = os.path.join(HERE, "_ref", "libpfref.so")
    if os.path.exists(path):
        return True
    if os.path.exists(os.path.join(REF_CHECKOUT, "src", "engine.cpp")):
        try:
            build()
        except RuntimeError:
            return False
        return os.path.exists(path)
    return False


def ref():
    """The reference's own functions (oracle/_ref/libpfref.so)."""
    global _ref
    if _ref is None:
        if not ref_available():
            raise FileNotFoundError("oracle/_ref/libpfref.so not built (no reference checkout)")
        L = C.CDLL(os.path.join(HERE, "_ref", "libpfref.so"))
        _sig(L, "pfref_quantize_activation_row", None, _f32p, _i8p, _f32p, u32)
        _sig(L, "pfref_dequant_q4_to_int8", None, _u8p, _i8p, u32)
        _sig(L, "pfref_dequant_q2_to_int8", None, _u8p, _i8p, u32)
        _sig(L, "pfref_dequant_ternary_to_int8", None, _u8p, _i8p, u32)
        _sig(L, "pfref_matmul_int8", None, _i8p, _i8p, _i32p, u32, u32, u32)
        _sig(L, "pfref_matmul_quantized", None, _f32p, _i8p, _f32p, u32, u32, u32, _f32p, vp)
        _sig(L, "pfref_rmsnorm", None, _f32p, _f32p, _f32p, u32)
        _sig(L, "pfref_softmax", None, _f32p, u32)
        _sig(L, "pfref_dot_product", f32, _f32p, _f32p, u32)
        _sig(L, "pfref_kv_create", vp, u32, u32, u32, u32, u32, u32, u32)
        _sig(L, "pfref_kv_destroy", None, vp)
        _sig(L, "pfref_kv_store", None, vp, u32, u32, u32, _f32p, _f32p)
        _sig(L, "pfref_kv_scores", u32, vp, u32, u32, _f32p, _f32p)
        _sig(L, "pfref_kv_weighted_sum", None, vp, u32, u32, _f32p, _f32p, u32)
        _sig(L, "pfref_kv_size", u32, vp)
        _sig(L, "pfref_kv_memory", u64, vp)
        _sig(L, "pfref_skip_create", vp, u32, u32, f32, u32)
        _sig(L, "pfref_skip_destroy", None, vp)
        _sig(L, "pfref_skip_should_skip", C.c_int, vp, u32, _f32p, u32)
        _sig(L, "pfref_skip_record", None, vp, u32, _f32p, u32)
        _sig(L, "pfref_skip_new_token", None, vp)
        _sig(L, "pfref_skip_is_anchor", C.c_int, vp)
        _sig(L, "pfref_skip_total", u32, vp)
        _sig(L, "pfref_skip_reset", None, vp)
        _sig(L, "pfref_skip_set_threshold", None, vp, f32)
        _sig(L, "pfref_mtp_create", vp, u32, u32, u32)
        _sig(L, "pfref_mtp_destroy", None, vp)
        _sig(L, "pfref_mtp_set_head", None, vp, u32, _u8p, _f32p, _u8p, _f32p, _u8p, _f32p)
        _sig(L, "pfref_mtp_forward", None, vp, _f32p, _f32p, u64, _f32p)
        _sig(L, "pfref_mtp_quantize_q4", None, _f32p, _u8p, _f32p, u32, u32)
        _sig(L, "pfref_mtp_argmax", i32, _f32p, u32)
        _sig(L, "pfref_mtp_speculative_accept", C.c_int, vp, i32, _f32p, u32)
        _sig(L, "pfref_quantize_matrix", u64, _f32p, u32, u32, C.c_int, vp)
        _sig(L, "pfref_squeeze_roundtrip", C.c_int, C.c_char_p, _f32p, u32, u32, C.c_int, _i8p,
             _f32p, _f32p)
        _sig(L, "pfref_write_squeeze_model", C.c_int, C.c_char_p, u32, u32, u32, u32, u32, u32, u32, u32, _f32p,
             np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS"))
        _sig(L, "pfref_load_block", C.c_int64, C.c_char_p, u32, u32, _i8p, _f32p, _f32p, C.c_int64)
        _sig(L, "pfref_write_test_engine_model", C.c_int, C.c_char_p)
        _sig(L, "pfref_write_literal_model", C.c_int, C.c_char_p, u32, u32, u32, u32, u32, u32, u32, u32, vp, vp,
             C.c_int)
        _sig(L, "pfref_literal_script", C.c_int64, C.c_char_p, u32, C.c_uint64, u32, C.c_char_p, C.c_int64)
        _sig(L, "pfref_engine_create", vp)
        _sig(L, "pfref_engine_destroy", None, vp)
        _sig(L, "pfref_seed_sampler", None, u32)
        _sig(L, "pfref_sample", i32, vp, _f32p, u32, f32, f32, u32, C.c_int)
        _sig(L, "pfref_sample_greedy", i32, vp, _f32p, u32)
        _sig(L, "pfref_sample_top_p", i32, vp, _f32p, u32, f32, f32)
        _sig(L, "pfref_sample_top_k", i32, vp, _f32p, u32, u32, f32)
        _ref = L
    return _ref
