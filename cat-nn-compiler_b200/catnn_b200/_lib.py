"""ctypes binding of libcatnn_b200.so (the C ABI in include/catnn_b200.h).

Loading fails loudly when the library is missing: there is no CPU or
PyTorch fallback for any operator of this package.
"""
import ctypes as C
import os

from .errors import raise_for

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libcatnn_b200.so")

I64, I32, U64, F32, F64, VP = C.c_int64, C.c_int, C.c_uint64, C.c_float, C.c_double, C.c_void_p
PP = C.POINTER(C.c_void_p)

# name -> argtypes (all return int status unless listed in _RESTYPE)
SIGNATURES = {
    "catnn_version": [],
    "catnn_last_error": [],
    "catnn_ctx_create": [I32, PP],
    "catnn_ctx_destroy": [VP],
    "catnn_ctx_set_stream": [VP, VP],
    "catnn_ctx_synchronize": [VP],
    "catnn_ctx_launch_count": [VP, C.POINTER(U64)],
    "catnn_malloc": [VP, C.c_size_t, PP],
    "catnn_free": [VP, VP],
    "catnn_upload": [VP, VP, VP, C.c_size_t],
    "catnn_download": [VP, VP, VP, C.c_size_t],
    "catnn_checksum_f32": [VP, VP, I64, C.POINTER(U64)],
    "catnn_gemm": [VP, I32, I32, I64, I64, I64, VP, I64, VP, I64, VP, I64, I32, I32, VP, I32, I32],
    "catnn_linear_fwd": [VP, VP, VP, VP, VP, I64, I64, I64, I32, I32],
    "catnn_linear_bwd": [VP, VP, VP, VP, VP, VP, VP, I64, I64, I64, I32],
    "catnn_lm_head_fwd": [VP, VP, VP, VP, I64, I64, I64, I32],
    "catnn_lm_head_bwd": [VP, VP, VP, VP, VP, VP, I64, I64, I64, I32],
    "catnn_relu_fwd": [VP, VP, VP, I64, I32],
    "catnn_gelu_fwd": [VP, VP, VP, I64, I32],
    "catnn_relu_bwd": [VP, VP, VP, VP, I64, I32],
    "catnn_gelu_bwd": [VP, VP, VP, VP, I64, I32],
    "catnn_add": [VP, VP, VP, VP, I64, I64, I32],
    "catnn_mul": [VP, VP, VP, VP, I64, I32],
    "catnn_softmax_fwd": [VP, VP, VP, I64, I64, I32],
    "catnn_softmax_bwd": [VP, VP, VP, VP, I64, I64, I32],
    "catnn_xent_fwdbwd": [VP, VP, VP, I64, I64, VP, VP, I32, I32],
    "catnn_xent_fwdbwd_noalloc": [VP, VP, VP, I64, I64, VP, VP, I32, I32],
    "catnn_mse_fwdbwd": [VP, VP, VP, I64, VP, VP],
    "catnn_layernorm_fwd": [VP, VP, VP, VP, VP, I64, I64, F32, I32],
    "catnn_layernorm_bwd": [VP, VP, VP, VP, VP, VP, VP, I64, I64, F32, I32],
    "catnn_rmsnorm_fwd": [VP, VP, VP, VP, I64, I64, F32, I32],
    "catnn_rmsnorm_bwd": [VP, VP, VP, VP, VP, VP, I64, I64, F32, I32],
    "catnn_embedding_fwd": [VP, VP, I64, VP, I64, I64, VP, I32],
    "catnn_embedding_bwd": [VP, VP, I64, VP, VP, I64, I64, I32],
    "catnn_rope": [VP, VP, I64, I64, I64, I64, F64, I32, I32],
    "catnn_attention_fwd": [VP, VP, VP, VP, VP, VP, I64, I64, I64, I64, I64, I32, I64, I32],
    "catnn_attention_bwd": [VP, VP, VP, VP, VP, VP, VP, VP, VP, VP, I64, I64, I64, I64, I64, I32, I64, I32],
    "catnn_mha_fwd": [VP, VP, VP, VP, VP, VP, VP, I64, I64, I64, I64, I32, I32],
    "catnn_mha_bwd": [VP, VP, VP, VP, VP, VP, VP, VP, VP, VP, VP, VP, I64, I64, I64, I64, I32, I32],
    "catnn_gqa_fwd": [VP, VP, VP, VP, VP, VP, VP, I64, I64, I64, I64, I64, I64, F64, I64, I32],
    "catnn_gqa_bwd": [VP, VP, VP, VP, VP, VP, VP, VP, VP, VP, VP, VP, I64, I64, I64, I64, I64, I64, F64, I64, I32],
    "catnn_router_topk": [VP, VP, I64, I64, I64, VP, VP],
    "catnn_moe_permute_map": [VP, VP, I64, I64, I64, I64, VP, VP, VP, VP],
    "catnn_moe_permute": [VP, VP, VP, I64, I64, I64, VP, I32],
    "catnn_moe_unpermute": [VP, VP, VP, VP, I64, I64, I64, VP, I32],
    "catnn_grouped_gemm": [VP, I32, I64, I64, I64, I64, VP, VP, VP, VP, I32, I32],
    "catnn_moe_expert_swiglu_fwd": [VP, VP, VP, VP, I64, I64, I64, I64, VP, VP],
    "catnn_moe_expert_swiglu_bwd": [VP, VP, VP, VP, VP, I64, I64, I64, I64, VP],
    "catnn_kernel_describe": [VP, C.c_char_p, I32, VP, VP],
    "catnn_swiglu_fwd": [VP, VP, VP, VP, VP, VP, I64, I64, I64, I32],
    "catnn_swiglu_bwd": [VP, VP, VP, VP, VP, VP, VP, VP, VP, VP, I64, I64, I64, I32],
    "catnn_moe_fwd": [VP, VP, VP, VP, VP, VP, VP, I64, I64, I64, I64, I64, I32],
    "catnn_moe_bwd": [VP, VP, VP, VP, VP, VP, VP, VP, VP, VP, VP, VP, I64, I64, I64, I64, I64, I32],
    "catnn_sgd": [VP, VP, VP, I64, F32, VP],
    "catnn_adam": [VP, VP, VP, VP, VP, I64, U64, F32, F32, F32, F32, I32, VP],
    "catnn_mlp_step": [VP, VP, VP, VP, VP, VP, VP, VP, I32, I64, I64, I64, I64, VP, VP, VP, VP, VP],
    "catnn_moe_trainer_create": [VP, VP, PP],
    "catnn_moe_trainer_destroy": [VP],
    "catnn_moe_trainer_param_count": [VP, C.POINTER(I64)],
    "catnn_moe_trainer_set_params": [VP, VP],
    "catnn_moe_trainer_get_params": [VP, VP],
    "catnn_moe_trainer_get_grads": [VP, VP],
    "catnn_moe_trainer_step": [VP, VP, VP, I32],
    "catnn_moe_trainer_step_host": [VP, VP, VP, I32],
    "catnn_moe_trainer_check": [VP],
    "catnn_moe_trainer_activation": [VP, I32, I64, VP],
    "catnn_moe_trainer_set_graphs": [VP, I32],
    "catnn_moe_trainer_set_profile": [VP, I32],
    "catnn_moe_trainer_timeline": [VP, C.POINTER(I64), I32, C.c_char_p, I64, C.POINTER(I32)],
    "catnn_moe_trainer_create_ep": [VP, VP, VP, PP],
    "catnn_comm_unique_id": [VP],
    "catnn_comm_create": [VP, I32, I32, VP, PP],
    "catnn_comm_destroy": [VP],
    "catnn_comm_rank": [VP, C.POINTER(I32), C.POINTER(I32)],
    "catnn_comm_set_timeout_ms": [VP, I64],
    "catnn_comm_allreduce": [VP, VP, I64, I32],
    "catnn_comm_all_to_all": [VP, VP, C.POINTER(I64), VP, C.POINTER(I64)],
    "catnn_comm_barrier": [VP],
    "catnn_comm_signal": [VP, I32, U64],
    "catnn_comm_wait": [VP, I32, U64],
    "catnn_comm_check": [VP],
}

_RESTYPE = {"catnn_last_error": C.c_char_p}

_lib = None


def load():
    """Load the library once; raise if it was never built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
            "(catnn_b200 has no CPU fallback)")
    lib = C.CDLL(LIB_PATH)
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPE.get(name, C.c_int)
    _lib = lib
    return lib


def last_error():
    return load().catnn_last_error().decode(errors="replace")


def call(name, *args):
    """Call an entry point and raise the matching CatError on failure."""
    rc = getattr(load(), name)(*args)
    if rc != 0:
        raise_for(rc, f"{name}: {last_error()}")
    return rc


def exported_symbols():
    return sorted(SIGNATURES)
