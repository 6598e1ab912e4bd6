"""Loader and ctypes signatures of libmoe_cuda.so (include/moe_cuda.h).

There is no fallback: if the CUDA library is missing or cannot be loaded this
module raises, so no code path silently computes on the CPU.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmoe_cuda.so")


class MoeConfigC(C.Structure):
    _fields_ = [("hidden", C.c_int), ("intermediate", C.c_int), ("n_experts", C.c_int), ("n_group", C.c_int),
                ("topk_group", C.c_int), ("top_k", C.c_int), ("routed_scale", C.c_float), ("rms_eps", C.c_float),
                ("n_layers", C.c_int), ("max_tokens", C.c_int)]


_vp = C.c_void_p
_fp = C.POINTER(C.c_float)
_ip = C.POINTER(C.c_int)

# name -> (restype, argtypes); kept in the order of include/moe_cuda.h
SIGNATURES = {
    "moe_get_unique_id": (C.c_int, [_vp]),
    "moe_create": (_vp, [C.POINTER(MoeConfigC), C.c_int, C.c_int, C.c_int, _vp]),
    "moe_destroy": (None, [_vp]),
    "moe_last_error": (C.c_char_p, [_vp]),
    "moe_stream": (_vp, [_vp]),
    "moe_rank": (C.c_int, [_vp]),
    "moe_world_size": (C.c_int, [_vp]),
    "moe_ep_peer_memory": (C.c_int, [_vp]),
    "moe_load_layer": (C.c_int, [_vp, C.c_int, _vp, _vp, _vp, C.c_int, _vp, _vp, _vp, _vp, _vp, C.c_int]),
    "moe_load_layer_shard": (C.c_int, [_vp, C.c_int, _vp, _vp, _vp, C.c_int, _vp, _vp, _vp, _vp, _vp, C.c_int]),
    "moe_shard_range": (C.c_int, [_vp, C.c_size_t, C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]),
    "moe_load_layer_packed": (C.c_int, [_vp, C.c_int, _vp, C.c_size_t, _vp, _vp, _vp, _vp, _vp, C.c_int]),
    "moe_init_layer_synthetic": (C.c_int, [_vp, C.c_int, C.c_uint64, C.c_int, C.c_double, C.c_double,
                                           C.c_double]),
    "moe_add_router_bias": (C.c_int, [_vp, C.c_int, _vp]),
    "moe_set_logit_bias": (C.c_int, [_vp, C.c_int, _vp]),
    "moe_set_norm_weight": (C.c_int, [_vp, C.c_int, _vp]),
    "moe_read_expert": (C.c_int, [_vp, C.c_int, C.c_int, _vp, C.c_size_t]),
    "moe_expert_bytes": (C.c_size_t, [_vp, C.c_int]),
    "moe_write_layer_packed": (C.c_int, [_vp, C.c_int, C.c_char_p]),
    "moe_load_dense_layer": (C.c_int, [_vp, C.c_int, C.c_int, _vp, C.c_int, _vp, C.c_int, _vp, C.c_int]),
    "moe_init_dense_synthetic": (C.c_int, [_vp, C.c_int, C.c_int, C.c_uint64, C.c_double]),
    "moe_read_dense_weight": (C.c_int, [_vp, C.c_int, C.c_int, _vp, C.c_size_t]),
    "moe_dense_forward": (C.c_int, [_vp, C.c_int, _vp, C.c_int, _vp]),
    "moe_dense_forward_device": (C.c_int, [_vp, C.c_int, _vp, C.c_int, _vp, _vp]),
    "moe_load_lm_head": (C.c_int, [_vp, C.c_int, _vp, C.c_int]),
    "moe_init_lm_head_synthetic": (C.c_int, [_vp, C.c_int, C.c_uint64, C.c_double]),
    "moe_read_lm_head": (C.c_int, [_vp, _vp, C.c_size_t]),
    "moe_lm_head": (C.c_int, [_vp, _vp, C.c_int, _vp]),
    "moe_lm_head_device": (C.c_int, [_vp, _vp, C.c_int, _vp, _vp]),
    "moe_sample": (C.c_int, [_vp, _vp, C.c_int, C.c_int, C.c_float, C.c_float, C.POINTER(C.c_uint32), _vp]),
    "moe_sample_device": (C.c_int, [_vp, _vp, C.c_int, C.c_int, C.c_float, C.c_float, C.c_uint32, _vp, _vp]),
    "moe_rng_advance": (C.c_uint32, [C.c_uint32, C.c_int]),
    "moe_forward": (C.c_int, [_vp, C.c_int, _vp, C.c_int, _vp, _vp, _vp]),
    "moe_forward_device": (C.c_int, [_vp, C.c_int, _vp, C.c_int, _vp, _vp, _vp, _vp]),
    "moe_check_error": (C.c_int, [_vp]),
    "moe_experts_forward": (C.c_int, [_vp, C.c_int, _vp, C.c_int, _vp, _vp, C.c_int, _vp]),
    "moe_experts_forward_device": (C.c_int, [_vp, C.c_int, _vp, C.c_int, _vp, _vp, C.c_int, _vp, _vp]),
    "moe_shared_forward": (C.c_int, [_vp, C.c_int, _vp, C.c_int, _vp]),
    "moe_route": (C.c_int, [_vp, _vp, _vp, C.c_int, _vp, _vp]),
    "moe_route_hidden_noalloc": (C.c_int, [C.POINTER(MoeConfigC), _vp, _vp, _vp, C.c_int, _vp, _vp, _vp]),
    "moe_forward_stack_device": (C.c_int, [_vp, C.c_int, C.c_int, _vp, C.c_int, _vp]),
    "moe_forward_stack": (C.c_int, [_vp, C.c_int, C.c_int, _vp, C.c_int]),
    "moe_prefill_device": (C.c_int, [_vp, C.c_int, _vp, C.c_int, _vp, _vp, _vp, _vp]),
    "moe_prefill": (C.c_int, [_vp, C.c_int, _vp, C.c_int, _vp, _vp, _vp]),
    "moe_dequantize_row_q4_K": (C.c_int, [_vp, _vp, C.c_size_t]),
    "moe_dequantize_row_q6_K": (C.c_int, [_vp, _vp, C.c_size_t]),
    "moe_kernel_launches": (C.c_uint64, [_vp]),
    "moe_reset_kernel_launches": (None, [_vp]),
    "moe_last_weight_bytes": (C.c_uint64, [_vp]),
    "moe_record_expert_hits": (C.c_int, [_vp, _vp]),
    "moe_set_timing": (C.c_int, [_vp, C.c_int]),
    "moe_get_timing": (C.c_int, [_vp, _vp, C.c_int]),
    "moe_get_timing_at": (C.c_int, [_vp, C.c_int, _vp, C.c_int]),
}

PHASES = ["router", "route", "dispatch", "gateup_tc", "gateup", "prep", "down_tc", "down", "combine_a2a", "output"]

_lib = None


def _bundled_nccl() -> str | None:
    """libnccl.so.2 of the nvidia-nccl wheel that torch links against.  The
    library dlopens NCCL on first expert-parallel use; pointing it at this
    copy keeps a later `import torch` in the same process working (both
    resolve the soname libnccl.so.2 to the same, newer, file)."""
    try:
        import importlib.util
        spec = importlib.util.find_spec("nvidia.nccl")
        for d in (spec.submodule_search_locations or []) if spec else []:
            p = os.path.join(d, "lib", "libnccl.so.2")
            if os.path.exists(p):
                return p
    except (ImportError, ValueError):
        pass
    return None


def load(build_if_missing: bool = False) -> C.CDLL:
    """Returns the loaded CUDA library; raises if it is not there."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        if build_if_missing:
            from . import build
            build.build()
        else:
            raise ImportError(f"libmoe_cuda.so not found at {LIB_PATH}: run `python -m flash_deepseek_b200.build` "
                              "(there is no CPU fallback)")
    if "MOE_NCCL_LIB" not in os.environ:
        nccl = _bundled_nccl()
        if nccl:
            os.environ["MOE_NCCL_LIB"] = nccl
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib
