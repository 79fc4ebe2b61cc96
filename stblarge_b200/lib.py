"""ctypes binding of libstbl_moe.so (include/stbl_moe.h, include/stbl_kernels.h, include/stbl_gguf.h,
include/stbl_io.h).

The reference drives its engine from Python through ctypes (stbl/run.py:37-47, stbl/test_kernels.py:25);
this module does the same for the B200 library.  There is no fallback: if the library is missing
the import of a layer fails with an error that says how to build it.
"""

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libstbl_moe.so")

P = ctypes.c_void_p
I = ctypes.c_int
F = ctypes.c_float
LL = ctypes.c_longlong
U32 = ctypes.c_uint32
U64 = ctypes.c_uint64


class MoEDesc(ctypes.Structure):
    _fields_ = [
        ("hidden", I), ("inter", I), ("n_experts", I), ("topk", I), ("n_groups", I), ("topk_groups", I),
        ("score_fn", I), ("route_scale", F), ("swiglu_limit", F), ("routed_fmt", I), ("shared_fmt", I),
        ("max_tokens", I), ("router_w", P), ("router_bias", P), ("routed_w", P * 3), ("routed_s", P * 3),
        ("routed_w_stride", LL * 3), ("routed_s_stride", LL * 3), ("shared_w", P * 3), ("shared_s", P * 3),
        ("n_slots", I), ("routed_s_blocked", I), ("act_q8", I),
    ]


class GgufTensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("type", U32), ("n_dims", U32), ("dims", U64 * 4), ("offset", U64),
                ("nbytes", U64), ("data", P)]


class CacheDesc(ctypes.Structure):
    _fields_ = [
        ("n_layers", I), ("n_experts", I), ("slots", I), ("fmt", I), ("hidden", I), ("inter", I),
        ("host_w", P * 3), ("host_s", P * 3), ("host_w_stride", LL * 3), ("host_s_stride", LL * 3),
        ("host_rows", LL),
    ]


class CacheFileDesc(ctypes.Structure):
    _fields_ = [("path", ctypes.c_char_p), ("offset", P), ("readers", I), ("direct", I), ("stage_experts", I)]


# every symbol the headers declare, with its C signature
SIGNATURES = {
    # include/stbl_moe.h
    "stbl_moe_create": (I, [ctypes.POINTER(MoEDesc), ctypes.POINTER(P), ctypes.c_char_p, I]),
    "stbl_moe_create_ep": (I, [ctypes.POINTER(MoEDesc), I, I, ctypes.POINTER(P), ctypes.c_char_p, I]),
    "stbl_moe_ep_handle": (I, [P, P]),
    "stbl_moe_ep_connect": (I, [P, P]),
    "stbl_moe_forward": (I, [P, P, I, P, P]),
    "stbl_moe_forward_host": (I, [P, P, I, P, P]),
    "stbl_moe_last_route": (I, [P, P, P, P, P, P]),
    "stbl_moe_last_scores": (I, [P, P]),
    "stbl_moe_last_acts": (I, [P, I, P, P, P]),
    "stbl_moe_set_expert": (I, [P, I, P, P, P]),
    "stbl_moe_forward_routed": (I, [P, P, I, P, P, P]),
    "stbl_moe_forward_block": (I, [P, P, P, F, P, P, P, I, I, P, P]),
    "stbl_cache_create": (I, [ctypes.POINTER(CacheDesc), ctypes.POINTER(P), ctypes.c_char_p, I]),
    "stbl_cache_layer_desc": (I, [P, ctypes.POINTER(MoEDesc)]),
    "stbl_moe_attach_cache": (I, [P, P, I]),
    "stbl_cache_stats": (I, [P, ctypes.POINTER(U64), ctypes.POINTER(U64), ctypes.POINTER(U64)]),
    "stbl_cache_info": (I, [P, ctypes.POINTER(I), ctypes.POINTER(U64)]),
    "stbl_cache_state": (I, [P, P, P]),
    "stbl_cache_destroy": (None, [P]),
    "stbl_cache_prefetch": (I, [P, I, P, I, I, P, P]),
    "stbl_cache_prefetch_stats": (I, [P, ctypes.POINTER(U64), ctypes.POINTER(U64), ctypes.POINTER(U64)]),
    "stbl_moe_attach_prefetch": (I, [P, P, I, I, P]),
    "stbl_cache_prefetch_counters": (I, [P, ctypes.POINTER(U64)]),
    "stbl_cache_create_file": (I, [ctypes.POINTER(CacheDesc), ctypes.POINTER(CacheFileDesc), ctypes.POINTER(P),
                                   ctypes.c_char_p, I]),
    "stbl_cache_file_stats": (I, [P, ctypes.POINTER(U64), ctypes.POINTER(U64), ctypes.POINTER(ctypes.c_double),
                                  ctypes.POINTER(I), ctypes.POINTER(U64)]),
    "stbl_cache_inject_read_error": (I, [P, ctypes.c_int64, I]),
    "stbl_cache_error": (ctypes.c_char_p, [P]),
    "stbl_mxfp4_from_gguf": (I, [P, I, I, P, P, P]),
    "stbl_moe_status": (I, [P, ctypes.POINTER(U32)]),
    "stbl_moe_set_timing": (I, [P, I]),
    "stbl_moe_timing": (I, [P, P, I]),
    "stbl_moe_stats": (None, [P, ctypes.POINTER(U64), ctypes.POINTER(U64), ctypes.POINTER(I)]),
    "stbl_moe_error": (ctypes.c_char_p, [P]),
    "stbl_moe_destroy": (None, [P]),
    "stbl_route_noalloc": (I, [P, P, P, I, I, I, I, I, I, I, F, P, P, P, P, P, P, ctypes.c_char_p, I]),
    "stbl_route_noalloc_status": (I, [ctypes.POINTER(U32)]),
    "stbl_gemv_mxfp4_q8": (I, [P, P, P, P, P, I, I, I, P]),
    # include/stbl_gguf.h
    "stbl_gguf_open": (I, [ctypes.c_char_p, ctypes.POINTER(P), ctypes.c_char_p, I]),
    "stbl_gguf_close": (None, [P]),
    "stbl_gguf_info": (I, [P, ctypes.POINTER(U32), ctypes.POINTER(U64), ctypes.POINTER(U64), ctypes.POINTER(U64)]),
    "stbl_gguf_tensor_at": (I, [P, U64, ctypes.POINTER(GgufTensor)]),
    "stbl_gguf_find": (I, [P, ctypes.c_char_p, ctypes.POINTER(GgufTensor)]),
    "stbl_gguf_kv_at": (I, [P, U64, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(U32)]),
    "stbl_gguf_u32": (I, [P, ctypes.c_char_p, ctypes.POINTER(U32)]),
    "stbl_gguf_f32": (I, [P, ctypes.c_char_p, ctypes.POINTER(F)]),
    "stbl_gguf_uints": (ctypes.c_int64, [P, ctypes.c_char_p, ctypes.POINTER(U64), ctypes.c_int64]),
    "stbl_gguf_str": (ctypes.c_int64, [P, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int64]),
    # include/stbl_io.h
    "stbl_reader_open": (I, [ctypes.c_char_p, I, I, ctypes.POINTER(P), ctypes.c_char_p, I]),
    "stbl_reader_region_bytes": (U64, [U64]),
    "stbl_reader_read": (I, [P, I, P, P, P, P]),
    "stbl_reader_stats": (I, [P, ctypes.POINTER(U64), ctypes.POINTER(U64), ctypes.POINTER(ctypes.c_double),
                              ctypes.POINTER(I)]),
    "stbl_reader_inject_error": (I, [P, ctypes.c_int64, I]),
    "stbl_reader_error": (ctypes.c_char_p, [P]),
    "stbl_reader_close": (None, [P]),
    # include/stbl_kernels.h
    "stbl_act_quant_fp8": (None, [P, I, P]),
    "stbl_round_bf16": (None, [P, I, P]),
    "stbl_gemv_fp8": (None, [P, P, P, P, I, I, I, P]),
    "stbl_gemv_mxfp4": (None, [P, P, P, I, I, P]),
    "stbl_gemv_mxfp4_batch": (None, [P, P, P, I, I, I, P]),
    "stbl_gemv_f32": (None, [P, P, P, I, I, I, P]),
    "stbl_sqrt_softplus": (None, [P, I, P]),
    "stbl_swiglu": (None, [P, P, P, F, F, I, P]),
    "stbl_swiglu_batch": (None, [P, P, P, P, I, F, I, P]),
    "stbl_axpy": (None, [P, P, F, I, P]),
}

_lib = None


def load():
    """The library, with argument types set.  Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m stblarge_b200.build` "
                               "(the MoE path has no CPU fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib
