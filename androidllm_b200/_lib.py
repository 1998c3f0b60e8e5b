"""ctypes binding of libandroidllm_b200.so (the pattern of androidllm/neon.py).

Unlike androidllm's optional NEON kernel there is no fallback: if the library
is missing or cannot load, importing this module raises.
"""
import ctypes
import os
import re

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libandroidllm_b200.so")
HEADER = os.path.join(os.path.dirname(_HERE), "include", "androidllm_b200.h")


class ALMError(RuntimeError):
    """A libandroidllm_b200 call returned a nonzero status."""

    def __init__(self, code, msg):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class ModelConfig(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int), ("layers", ctypes.c_int), ("heads", ctypes.c_int),
                ("kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int),
                ("intermediate", ctypes.c_int), ("vocab", ctypes.c_int),
                ("max_len", ctypes.c_int), ("rms_eps", ctypes.c_float)]


class ProjSrc(ctypes.Structure):
    _fields_ = [("packed_host", ctypes.c_void_p), ("scale_host", ctypes.c_void_p),
                ("bits", ctypes.c_int), ("block", ctypes.c_int), ("out", ctypes.c_int),
                ("in_", ctypes.c_int), ("in_real", ctypes.c_int)]


_P = ctypes.c_void_p
_I = ctypes.c_int
_PP = ctypes.POINTER(ctypes.c_void_p)
_PI32 = ctypes.POINTER(ctypes.c_int32)

# name -> argtypes (all return int status unless listed in _RESTYPE)
SIGNATURES = {
    "alm_last_error": [],
    "alm_abi_version": [],
    "alm_ctx_create": [_I, _PP],
    "alm_ctx_destroy": [_P],
    "alm_ctx_sync": [_P],
    "alm_ctx_set_persistent": [_P, _I],
    "alm_ctx_set_gemv_layout": [_P, _I],
    "alm_ctx_set_cluster_forward": [_P, _I],
    "alm_nccl_unique_id": [_P],
    "alm_ctx_init_tp": [_P, _I, _I, _P],
    "alm_dev_alloc": [_P, ctypes.c_size_t, _PP],
    "alm_dev_free": [_P, _P],
    "alm_copy_h2d": [_P, _P, _P, ctypes.c_size_t],
    "alm_copy_d2h": [_P, _P, _P, ctypes.c_size_t],
    "alm_qweight_upload": [_P, _P, _P, _I, _I, _I, _I, _I, _PP],
    "alm_qweight_free": [_P],
    "alm_qweight_set_split": [_P, _I, _I],
    "alm_qweight_get_split": [_P, _PI32, _PI32, _PI32],
    "alm_qweight_dequant": [_P, _P, _P],
    "alm_qmatmul": [_P, _P, _P, _I, _I, _P, _I],
    "alm_qmatmul_noalloc": [_P, _P, _P, _I, _I, _P, _I],
    "alm_matmul_f16_f16": [_P, _P, _P, _P, _I, _I, _I],
    "alm_model_create": [_P, ctypes.POINTER(ModelConfig), _P, _PP],
    "alm_model_destroy": [_P],
    "alm_model_set_layer": [_P, _I, ctypes.POINTER(ProjSrc), _P, _P],
    "alm_model_set_embed": [_P, _P, _P, _I, _I],
    "alm_model_set_final_norm": [_P, _P],
    "alm_model_set_head": [_P, ctypes.POINTER(ProjSrc)],
    "alm_model_finalize": [_P],
    "alm_model_cluster_forward": [_P, _PI32],
    "alm_model_set_tp": [_P, _I, _I],
    "alm_kv_create": [_P, _P, _I, _I, _PP],
    "alm_kv_destroy": [_P],
    "alm_kv_zero": [_P],
    "alm_kv_read": [_P, _I, _I, _I, _P, _P],
    "alm_kv_write": [_P, _I, _I, _I, _P, _P],
    "alm_layer_forward": [_P, _I, _P, _P, _I, _I, _P],
    "alm_head_logits": [_P, _P, _I, _P, _P],
    "alm_forward": [_P, _P, _P, _I, _I, _P, _P],
    "alm_prefill": [_P, _P, _P, _I, _I],
    "alm_prefill_slot": [_P, _P, _I, _P, _I, _I],
    "alm_ctx_set_attn_fused": [_P, _I],
    "alm_tp_p2p_open": [_P, _I, _P],
    "alm_tp_p2p_connect": [_P, _P],
    "alm_ctx_set_tp_p2p": [_P, _I],
    "alm_model_sample_rows": [_P, _I, _I, ctypes.c_float, ctypes.c_float, ctypes.c_float, _P, _P],
    "alm_forward_seqs": [_P, _P, _I, _P, _P, _P, _P, _P, _P],
    "alm_kv_create_slots": [_P, _P, _I, _I, _I, _P],
    "alm_kv_read_slot": [_P, _I, _I, _I, _I, _P, _P],
    "alm_kv_set_pages": [_P, _I, _P, _I],
    "alm_ctx_set_dense_prefill": [_P, _I],
    "alm_model_dense_prefill": [_P, _P],
    "alm_model_max_pass_rows": [_P, _P],
    "alm_forward_trace": [_P, _P, _P, _I, _I, _P, _I, _P, _P],
    "alm_spec_create": [_P, _P, _P, _P, _I, _PP],
    "alm_spec_destroy": [_P],
    "alm_spec_begin": [_P, ctypes.c_int32, _I],
    "alm_spec_begin_prev": [_P, ctypes.c_int32, ctypes.c_int32, _I],
    "alm_spec_set_draft_refresh": [_P, _I],
    "alm_spec_run": [_P, _I, _P, _P, _P],
    "alm_spec_state": [_P, _PI32, _PI32],
    "alm_spec_kernel_count": [_P, _PI32],
    "alm_spec_set_sampling": [_P, ctypes.c_float, ctypes.c_float, ctypes.c_float],
    "alm_spec_set_uniforms": [_P, _P, _I],
    "alm_spec_set_rejection": [_P, _I],
    "alm_probs": [_P, _P, _I, _I, ctypes.c_float, ctypes.c_float, _P],
    "alm_accept": [_P, _P, _P, _P, _I, _I, ctypes.c_float, ctypes.c_float, _P, _P, _PI32],
    "alm_spec_uniforms_used": [_P, _PI32],
    "alm_sample": [_P, _P, _I, _I, ctypes.c_float, ctypes.c_float, ctypes.c_float, _P, _P],
    "alm_model_sample": [_P, _I, ctypes.c_float, ctypes.c_float, ctypes.c_float, _P, _P],
    "alm_profiler_range": [_I],
    "alm_spec_bench": [_P, _I, ctypes.POINTER(ctypes.c_float), _PI32],
    "alm_spec_profile": [_P, _I, _P, _P, _P, _PI32],
    "alm_bench_qmatmul": [_P, _PP, _I, _P, _I, _P, _I, ctypes.POINTER(ctypes.c_float)],
}
_RESTYPE = {"alm_last_error": ctypes.c_char_p}


def header_symbols(path=HEADER):
    """Function names declared in include/androidllm_b200.h."""
    with open(path, encoding="utf-8") as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(alm_[a-z0-9_]+)\s*\(", text)))


def _load():
    if not os.path.exists(LIB_PATH):
        raise OSError(f"{LIB_PATH} not found: build it with `python -m androidllm_b200.build`")
    lib = ctypes.CDLL(LIB_PATH)
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPE.get(name, ctypes.c_int)
    return lib


lib = _load()


def check(rc):
    if rc != 0:
        raise ALMError(rc, lib.alm_last_error().decode("utf-8", "replace"))
    return rc


def ptr(a):
    """Host pointer of a C-contiguous numpy array (or None)."""
    if a is None:
        return None
    if not a.flags["C_CONTIGUOUS"]:
        raise ValueError("array must be C-contiguous")
    return a.ctypes.data_as(ctypes.c_void_p)
