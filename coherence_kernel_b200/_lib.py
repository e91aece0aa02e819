"""ctypes binding of libck_b200.so (the C ABI in include/ck_b200.h and include/fk_cuda_carrier.h).

The library is the product: there is no fallback.  If it is missing or cannot be loaded the
import of any op raises, loudly.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libck_b200.so")

_p = ctypes.c_void_p
_u32 = ctypes.c_uint32
_u64 = ctypes.c_uint64
_i32 = ctypes.c_int
_f = ctypes.c_float
_ll = ctypes.c_longlong
_sz = ctypes.c_size_t


class MoeConfig(ctypes.Structure):
    """ck_moe_config (include/ck_b200.h)."""
    _fields_ = [("hidden", _u32), ("inter", _u32), ("n_experts", _u32), ("n_shared", _u32), ("nsel", _u32),
                ("mode", _u32), ("ngroups", _u32), ("topk_groups", _u32), ("wscale", _f), ("tau", _f)]


class DecodeConfig(ctypes.Structure):
    """ck_decode_config (include/ck_b200.h)."""
    _fields_ = [("hidden", _u32), ("max_tokens", _u32), ("eps", _f), ("moe", MoeConfig)]


# name -> (restype, argtypes); every symbol include/*.h declares
SIGNATURES = {
    "ck_last_error": (ctypes.c_char_p, []),
    "ck_device_ok": (_i32, []),
    "ck_q8_0_dequant_f32": (_i32, [_p, _p, _u64, _u64, _p]),
    "ck_q4k_dequant_f32": (_i32, [_p, _p, _u64, _u64, _p]),
    "ck_q4k_dequant_bf16": (_i32, [_p, _p, _u64, _u64, _p]),
    "ck_q8_0_matvec_f32": (_i32, [_p, _p, _p, _u32, _u32, _p]),
    "ck_q4k_matvec_f32": (_i32, [_p, _p, _p, _u32, _u32, _p]),
    "ck_matvec_ordered_f32": (_i32, [_i32, _p, _p, _p, _u32, _u32, _p]),
    "ck_q4k_matvec_f32_group": (_i32, [_u32, _p, _p, _p, _u32, _u32, _p]),
    "ck_q4k_matmul_batch_f32": (_i32, [_p, _p, _p, _u32, _u32, _u32, _p]),
    "ck_q6k_dequant_f32": (_i32, [_p, _p, _u64, _u64, _p]),
    "ck_q6k_matvec_f32": (_i32, [_p, _p, _p, _u32, _u32, _p]),
    "ck_q6k_matmul_batch_f32": (_i32, [_p, _p, _p, _u32, _u32, _u32, _p]),
    "ck_q6k_matvec_part_f32": (_i32, [_p, _p, _p, _u32, _u32, _u32, _p]),
    "ck_q4k_gemm_workspace_bytes": (_sz, [_u32]),
    "ck_q4k_gemm_bf16": (_i32, [_p, _p, _p, _u32, _u32, _u32, _p, _sz, _p]),
    "ck_q4k_gemm_status": (_i32, [_u32, _p, _p]),
    "ck_q4k_gemm_bf16_noalloc": (_i32, [_p, _p, _p, _u32, _u32, _u32, _p]),
    "ck_q4k_gemm_bf16_noalloc_status": (_i32, [_p]),
    "ck_f16_matvec_f32": (_i32, [_p, _p, _p, _u32, _u32, _p]),
    "ck_route_softmax_f32": (_i32, [_p, _p, _p, _u32, _u32, _u32, _i32, _p]),
    "ck_route_dsv4_f32": (_i32, [_p, _p, _p, _p, _u32, _u32, _f, _u32, _p]),
    "ck_scale_f32": (_i32, [_p, _p, _f, _u32, _p]),
    "ck_axpy_f32": (_i32, [_p, _p, _f, _u32, _p]),
    "ck_swiglu_f32": (_i32, [_p, _p, _p, _u32, _f, _f, _p]),
    "ck_moe_workspace_bytes": (_sz, [ctypes.POINTER(MoeConfig), _u32]),
    "ck_moe_layer_bf16": (_i32, [ctypes.POINTER(MoeConfig), _p, _u32, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
                                 _p, _sz, _p]),
    "ck_moe_layer_status": (_i32, [ctypes.POINTER(MoeConfig), _u32, _p, _p]),
    "ck_moe_route_workspace_bytes": (_sz, [ctypes.POINTER(MoeConfig), _u32]),
    "ck_moe_route": (_i32, [ctypes.POINTER(MoeConfig), _p, _u32, _p, _p, _p, _p, _p, _p, _sz, _p]),
    "ck_router_exact_logits": (_i32, [_p, _p, _p, _p, _u32, _u32, _p, _p, _p]),
    "ck_moe_route_flagged": (_i32, [ctypes.POINTER(MoeConfig), _u32, _p, _p]),
    "ck_moe_permute_workspace_bytes": (_sz, [_u32, _u32, _u32]),
    "ck_moe_max_tiles": (_u32, [_u32, _u32, _u32, _u32]),
    "ck_moe_permute": (_i32, [_p, _p, _p, _u32, _u32, _u32, _u32, _u32, _i32, _p, _p, _p, _p, _p, _p, _p, _p]),
    "ck_moe_expert_gemm": (_i32, [_i32, _p, _p, _p, _p, _u64, _u32, _u32, _p, _u32, _p, _u32, _p, _p, _p, _u32, _u32,
                                  _u32, _i32, _p, _p]),
    "ck_moe_expert_gemm_bounded": (_i32, [_i32, _p, _p, _p, _p, _u64, _u32, _u32, _p, _u32, _p, _u32, _p, _p, _p,
                                          _u32, _u32, _u32, _i32, _u32, _p, _p]),
    "ck_moe_expert_gemm_rows": (_i32, [_p, _u64, _u32, _p, _u32, _p, _u32, _p, _p, _u32, _u32, _u32, _i32, _p, _p]),
    "ck_moe_combine": (_i32, [_p, _p, _p, _p, _u32, _u32, _u32, _u32, _i32, _p, _p, _p]),
    "ck_token_tiles": (_i32, [_p, _p, _u32, _p]),
    "ck_token_tiles_n": (_i32, [_p, _p, _u32, _u32, _p]),
    "ck_gather_rows": (_i32, [_p, _p, _p, _u32, _u32, _p]),
    "ck_ep_dispatch_plan": (_i32, [_p, _p, _u32, _u32, _u32, _u32, _p, _p, _p, _p, _p, _p]),
    "ck_wait_selftest": (_i32, [_u64, _p, _p, _p]),
    "ck_ep_arena_alloc": (_i32, [_sz, _p]),
    "ck_ep_arena_free": (_i32, [_p]),
    "ck_ipc_get_handle": (_i32, [_p, _p]),
    "ck_ipc_open_handle": (_i32, [_p, _p]),
    "ck_ipc_close": (_i32, [_p]),
    "ck_ep_peer_status": (_i32, [_p, _p]),
    "ck_ep_peer_begin": (_i32, [_p, _p]),
    "ck_ep_peer_dispatch": (_i32, [_p, _p, _p, _p, _p, _u32, _p]),
    "ck_ep_peer_signal": (_i32, [_p, _i32, _p]),
    "ck_ep_peer_wait": (_i32, [_p, _i32, _u64, _p]),
    "ck_ep_peer_return": (_i32, [_p, _p, _p, _p, _p, _p]),
    "ck_ep_peer_return_rows": (_i32, [_p, _p, _p, _p, _p, _p]),
    "ck_ep_group_create": (_p, [ctypes.POINTER(MoeConfig), _u32, _p, _u32]),
    "ck_ep_group_load": (_i32, [_p, _p, _p, _p, _p, _p, _p, _p, _p]),
    "ck_ep_group_forward": (_i32, [_p, _p, _u32, _p, _p, _p, _p, _p]),
    "ck_ep_group_status": (_i32, [_p]),
    "ck_ep_group_destroy": (None, [_p]),
    "ck_decode_step_workspace_bytes": (_sz, [ctypes.POINTER(DecodeConfig)]),
    "ck_decode_step_create": (_p, [ctypes.POINTER(DecodeConfig)] + [_p] * 15 + [_sz]),
    "ck_decode_step_run": (_i32, [_p, _p, _p, _p, _p, _u32, _p]),
    "ck_decode_step_capture": (_i32, [_p, _p, _p, _p, _p, _u32, _p]),
    "ck_decode_step_replay": (_i32, [_p, _p]),
    "ck_decode_step_status": (_i32, [_p, _u32, _p]),
    "ck_decode_step_destroy": (None, [_p]),
    # the handle door
    "fk_metal_pipeline_external": (_ll, [ctypes.c_char_p, _ll, ctypes.c_char_p, _ll]),
    "fk_metal_buf_alloc_external": (_ll, [_ll]),
    "fk_metal_buf_from_file_external": (_ll, [ctypes.c_char_p, _ll, _ll, _ll]),
    "fk_metal_buf_write_external": (_ll, [_ll, _ll, ctypes.c_char_p, _ll]),
    "fk_metal_enqueue_external": (_ll, [_ll, ctypes.c_char_p, _ll, _ll]),
    "fk_metal_sync_external": (_ll, []),
    "fk_metal_buf_read_external": (_ll, [_ll, _ll, _ll, ctypes.c_char_p, _ll]),
    "fk_metal_status_external": (_ll, [ctypes.c_char_p, _ll]),
    "fk_metal_batch_concurrent_external": (_ll, []),
    "fk_metal_buf_free_external": (_ll, [_ll]),
    "fk_metal_submit_external": (_ll, []),
    "fk_metal_fence_wait_external": (_ll, [_ll]),
    "fk_cuda_go_external": (_ll, [_p, _p, _p, _u32, _u32, ctypes.c_char_p, _ll]),
    "fk_cuda_matvec_f32_external": (_ll, [_p, _p, _p, _u32, _u32]),
    "fk_cuda_matvec_fixture_external": (_ll, []),
    "fk_metal_matvec_fixture_external": (_ll, [ctypes.c_char_p, _ll]),
    "fk_metal_matvec_f32_external": (_ll, [ctypes.c_char_p, _ll, ctypes.c_char_p, _ll, ctypes.c_char_p, _ll,
                                           ctypes.c_char_p, _ll]),
}

_lib = None


class CKError(RuntimeError):
    pass


def load():
    """Load libck_b200.so; raise if it is absent (build it with ``python -m coherence_kernel_b200.build``)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise CKError(f"{LIB_PATH} is missing: the CUDA kernels are not built "
                          "(python -m coherence_kernel_b200.build)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int, what: str = ""):
    if rc != 0:
        msg = load().ck_last_error().decode(errors="replace")
        raise CKError(f"{what or 'ck call'} failed ({rc}): {msg}")
