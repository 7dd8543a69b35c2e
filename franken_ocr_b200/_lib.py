"""ctypes binding of ``libfocr_cuda.so`` (the C ABI in ``include/focr_cuda.h``).

The library is the product: there is no CPU fallback.  If the shared object is
missing, importing this module raises immediately.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libfocr_cuda.so"

FOCR_OK = 0
FOCR_E_SHAPE = -1
FOCR_E_ARG = -2
FOCR_E_CUDA = -3
FOCR_E_ALLOC = -4
FOCR_E_ROUTE = -5
FOCR_E_TIMEOUT = -6
FOCR_E_UNSUPPORTED = -7
MEM_HOST = 0
MEM_DEVICE = 1

# Every symbol declared in include/focr_cuda.h.
EXPORTS = [
    "focr_last_error", "focr_tier_string", "focr_igemm_s8s8", "focr_igemm_u8s8",
    "focr_igemm_s4s8_packed", "focr_quantize_rows_i8", "focr_gemv_i8", "focr_gemv_i8_noalloc",
    "focr_moe_create", "focr_moe_destroy", "focr_moe_route", "focr_moe_forward",
    "focr_moe_decode", "focr_moe_prefill", "focr_moe_forward_rows", "focr_moe_combine",
    "focr_lmhead_create", "focr_lmhead_create_s4", "focr_lmhead_destroy", "focr_lmhead_top1",
    "focr_top1_combine", "focr_selftest", "focr_trace_set", "focr_rms_norm", "focr_rope_apply",
    "focr_attention_decode", "focr_linear_i8", "focr_swiglu", "focr_add",
    "focr_attention_prefill", "focr_rope_table", "focr_decode_prologue", "focr_rope_apply_at",
    "focr_ring_write", "focr_attention_decode_at", "focr_add_rms_norm",
    "focr_igemm_status", "focr_status_check",
    "focr_nccl_unique_id", "focr_comm_create", "focr_comm_destroy", "focr_top1_allgather",
    "focr_ep_create", "focr_ep_destroy", "focr_ep_ipc_handle", "focr_ep_connect",
    "focr_ep_connect_comm", "focr_ep_connect_local", "focr_ep_forward", "focr_ep_dispatch",
    "focr_ep_experts", "focr_ep_combine", "focr_ep_decode", "focr_ep_status",
    "focr_decoder_create", "focr_decoder_destroy", "focr_decoder_prefill", "focr_decoder_generate",
    "focr_rms_norm_linear_i8", "focr_rope_ring_at",
]


class FocrError(RuntimeError):
    """A non-zero status from the C ABI; ``.code`` is the FOCR_E_* value."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


if not LIB_PATH.exists():
    raise ImportError(
        f"{LIB_PATH} is missing: build it with `python franken_ocr_b200/build.py` "
        "(the CUDA library is required; there is no CPU fallback)")

lib = C.CDLL(str(LIB_PATH))

vp = C.c_void_p
sz = C.c_size_t
i32 = C.c_int


class MoeConfig(C.Structure):
    _fields_ = [
        ("hidden", C.c_uint32), ("inter", C.c_uint32), ("n_experts", C.c_uint32),
        ("topk", C.c_uint32), ("shared_inter", C.c_uint32), ("norm_topk_prob", C.c_int32),
        ("routed_scaling_factor", C.c_float), ("group", C.c_uint32),
        ("expert_begin", C.c_uint32), ("expert_count", C.c_uint32),
        ("max_tokens", C.c_uint32),
    ]


class MoeWeights(C.Structure):
    _fields_ = [(n, vp) for n in (
        "router", "gate_w", "gate_s", "up_w", "up_s", "down_w", "down_s",
        "gate_p", "gate_gs", "up_p", "up_gs", "down_p", "down_gs",
        "sh_gate_w", "sh_gate_s", "sh_up_w", "sh_up_s", "sh_down_w", "sh_down_s")]


class DecoderConfig(C.Structure):
    _fields_ = [
        ("hidden", C.c_uint32), ("heads", C.c_uint32), ("head_dim", C.c_uint32),
        ("n_layers", C.c_uint32), ("vocab", C.c_uint32), ("max_prefill", C.c_uint32),
        ("ring_window", C.c_uint32), ("rope_theta", C.c_float), ("rms_eps", C.c_float),
        ("moe", MoeConfig),
    ]


class DecoderLayerWeights(C.Structure):
    _fields_ = [(n, vp) for n in (
        "input_ln", "post_ln", "q_w", "k_w", "v_w", "o_w", "q_s", "k_s", "v_s", "o_s", "moe")] + [
        ("dense_inter", C.c_uint32)] + [(n, vp) for n in (
            "gate_w", "up_w", "down_w", "gate_s", "up_s", "down_s")]


class DecoderWeights(C.Structure):
    _fields_ = [("layers", C.POINTER(DecoderLayerWeights))] + [
        (n, vp) for n in ("final_norm", "lm_w", "lm_s", "embed")]


lib.focr_last_error.restype = C.c_char_p
lib.focr_tier_string.restype = C.c_char_p
for _name in ("focr_igemm_s8s8", "focr_igemm_u8s8"):
    getattr(lib, _name).argtypes = [vp, sz, vp, sz, sz, sz, sz, vp, sz, i32, vp]
lib.focr_igemm_s4s8_packed.argtypes = [vp, sz, vp, sz, vp, sz, sz, sz, sz, sz, vp, sz, i32, vp]
lib.focr_igemm_status.argtypes = [C.POINTER(i32), i32]
lib.focr_status_check.argtypes = [i32]
lib.focr_quantize_rows_i8.argtypes = [vp, sz, sz, i32, vp, vp, i32, vp]
lib.focr_gemv_i8.argtypes = [vp, sz, sz, vp, vp, sz, vp, i32, vp]
lib.focr_gemv_i8_noalloc.argtypes = [vp, sz, sz, vp, vp, sz, vp, vp]
lib.focr_moe_create.argtypes = [C.POINTER(MoeConfig), C.POINTER(MoeWeights), C.POINTER(vp)]
lib.focr_moe_destroy.argtypes = [vp]
lib.focr_moe_route.argtypes = [vp, vp, sz, vp, vp, i32, vp]
lib.focr_moe_forward.argtypes = [vp, vp, sz, vp, vp, vp, i32, vp]
lib.focr_moe_decode.argtypes = [vp, vp, sz, vp, vp, vp, i32, vp]
lib.focr_moe_prefill.argtypes = [vp, vp, sz, vp, vp, vp, i32, vp]
lib.focr_moe_combine.argtypes = [vp, vp, vp, sz, sz, sz, vp, vp]
lib.focr_moe_forward_rows.argtypes = [vp, vp, sz, vp, vp, vp, sz, vp]
lib.focr_nccl_unique_id.argtypes = [vp]
lib.focr_comm_create.argtypes = [vp, C.c_uint32, C.c_uint32, C.POINTER(vp)]
lib.focr_comm_destroy.argtypes = [vp]
lib.focr_top1_allgather.argtypes = [vp, vp, vp, sz, vp, vp, vp]
lib.focr_ep_create.argtypes = [C.POINTER(MoeConfig), C.POINTER(MoeWeights), C.c_uint32,
                               C.c_uint32, C.POINTER(vp)]
lib.focr_ep_destroy.argtypes = [vp]
lib.focr_ep_ipc_handle.argtypes = [vp, vp]
lib.focr_ep_connect.argtypes = [vp, vp]
lib.focr_ep_connect_comm.argtypes = [vp, vp]
lib.focr_ep_connect_local.argtypes = [vp, sz]
lib.focr_ep_forward.argtypes = [vp, vp, sz, vp, vp, vp, vp]
lib.focr_ep_dispatch.argtypes = [vp, vp, sz, vp, vp, vp]
lib.focr_ep_experts.argtypes = [vp, vp]
lib.focr_ep_combine.argtypes = [vp, vp, vp]
lib.focr_ep_decode.argtypes = [vp, vp, sz, vp, vp, vp, vp]
lib.focr_ep_status.argtypes = [vp, C.POINTER(i32)]
lib.focr_lmhead_create.argtypes = [vp, vp, sz, sz, sz, sz, C.POINTER(vp)]
lib.focr_lmhead_create_s4.argtypes = [vp, vp, sz, sz, sz, sz, sz, C.POINTER(vp)]
lib.focr_lmhead_destroy.argtypes = [vp]
lib.focr_lmhead_top1.argtypes = [vp, vp, sz, vp, vp, vp, i32, vp]
lib.focr_top1_combine.argtypes = [vp, vp, sz, sz, vp]
lib.focr_selftest.argtypes = [C.c_char_p, sz, C.POINTER(i32)]
lib.focr_trace_set.argtypes = [vp, vp, sz]
lib.focr_rms_norm.argtypes = [vp, sz, sz, vp, C.c_float, vp, i32, vp]
lib.focr_rope_apply.argtypes = [vp, sz, sz, sz, vp, vp, i32, vp]
lib.focr_attention_decode.argtypes = [vp, vp, vp, sz, sz, vp, vp, sz, sz, sz, sz, vp, i32, vp]
lib.focr_linear_i8.argtypes = [vp, sz, sz, vp, vp, sz, i32, vp, i32, vp]
lib.focr_swiglu.argtypes = [vp, sz, sz, vp, i32, vp]
lib.focr_add.argtypes = [vp, vp, sz, vp, i32, vp]
lib.focr_attention_prefill.argtypes = [vp, vp, vp, sz, sz, sz, vp, i32, vp]
lib.focr_rope_table.argtypes = [vp, sz, sz, C.c_float, vp, vp]
lib.focr_decode_prologue.argtypes = [vp, vp, vp, sz, sz, sz, vp, sz, vp, vp]
lib.focr_rope_ring_at.argtypes = [vp, sz, sz, vp, vp, vp, vp, sz, vp, vp]
lib.focr_rms_norm_linear_i8.argtypes = [vp, vp, sz, vp, C.c_float, vp, vp, vp, sz, vp, vp]
lib.focr_decoder_create.argtypes = [C.POINTER(DecoderConfig), C.POINTER(DecoderWeights),
                                    C.POINTER(vp)]
lib.focr_decoder_destroy.argtypes = [vp]
lib.focr_decoder_prefill.argtypes = [vp, vp, sz, vp, i32, vp]
lib.focr_decoder_generate.argtypes = [vp, vp, sz, sz, vp, i32, vp]
lib.focr_rope_apply_at.argtypes = [vp, sz, sz, vp, vp, vp, vp]
lib.focr_ring_write.argtypes = [vp, vp, sz, sz, vp, vp, sz, vp, vp]
lib.focr_add_rms_norm.argtypes = [vp, vp, sz, sz, vp, C.c_float, vp, vp, vp]
lib.focr_attention_decode_at.argtypes = [vp, vp, vp, sz, sz, vp, vp, sz, sz, sz, vp, vp, vp]
STATE_POS, STATE_RING_LEN, STATE_RING_POS, STATE_SLOT, STATE_NEXT_POS, STATE_STEP = range(6)
STATE_ERROR, STATE_WORDS = 6, 8


def check(rc: int) -> None:
    if rc != FOCR_OK:
        raise FocrError(rc, lib.focr_last_error().decode(errors="replace"))
