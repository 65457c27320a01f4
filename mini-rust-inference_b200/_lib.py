"""ctypes binding of libmri_gpu.so (include/mri_gpu.h).

The library is built in-tree by build.py.  Loading fails loudly when the
shared object cannot be built or loaded: there is no CPU fallback.
"""
import ctypes
import os
import threading

from . import build as _build

OK = 0
INVALID_SHAPE = 1
SHAPE_MISMATCH = 2
CUDA_ERROR = 3
COMM_ERROR = 4
TIMEOUT = 5
INVALID_ARGUMENT = 6

PER_TENSOR = 0
PER_ROW = 1

_P = ctypes.c_void_p
_SZ = ctypes.c_size_t
_I = ctypes.c_int
_F = ctypes.c_float
_PP = ctypes.POINTER(ctypes.c_void_p)

# name -> (restype, argtypes); mirrors include/mri_gpu.h one to one.
SIGNATURES = {
    "mri_abi_version": (_I, []),
    "mri_last_error": (ctypes.c_char_p, []),
    "mri_ctx_create": (_I, [_I, _PP]),
    "mri_ctx_create_on_stream": (_I, [_I, _P, _PP]),
    "mri_ctx_destroy": (_I, [_P]),
    "mri_ctx_synchronize": (_I, [_P]),
    "mri_ctx_stream": (_P, [_P]),
    "mri_ctx_check_device_status": (_I, [_P]),
    "mri_ctx_launch_count": (ctypes.c_uint64, [_P]),
    "mri_ctx_set_option": (_I, [_P, _I, _I]),
    "mri_ctx_get_option": (_I, [_P, _I, ctypes.POINTER(_I)]),
    "mri_qmatrix_upload": (_I, [_P, _P, _P, _SZ, _SZ, _PP]),
    "mri_qmatrix_upload_rows": (_I, [_P, _P, _P, _SZ, _SZ, _SZ, _SZ, _PP]),
    "mri_qmatrix_free": (_I, [_P]),
    "mri_qmatrix_dims": (_I, [_P, ctypes.POINTER(_SZ), ctypes.POINTER(_SZ)]),
    "mri_q8_0_upload": (_I, [_P, _P, _SZ, _SZ, _SZ, _PP]),
    "mri_q8_0_free": (_I, [_P]),
    "mri_q4_0_upload": (_I, [_P, _P, _SZ, _SZ, _SZ, _PP]),
    "mri_q4_0_free": (_I, [_P]),
    "mri_quantize_symmetric": (_I, [_P, _P, _SZ, _SZ, _I, _P, _P]),
    "mri_matmul_int8": (_I, [_P, _P, _SZ, _F, _P, _SZ, _P, _P]),
    "mri_matmul_int8_dscale": (_I, [_P, _P, _SZ, _P, _I, _P, _SZ, _P, _P]),
    "mri_matmul_int8_from_f32": (_I, [_P, _P, _SZ, _SZ, _P, _P]),
    "mri_matmul_int8_from_f32_g": (_I, [_P, _P, _SZ, _SZ, _I, _P, _P]),
    "mri_matmul_q8_0_direct": (_I, [_P, _P, _SZ, _SZ, _P, _P]),
    "mri_matmul_q4_0_dequant": (_I, [_P, _P, _SZ, _SZ, _P, _P]),
    "mri_host_quantize_symmetric": (_I, [_P, _P, _SZ, _SZ, _I, _P, _P]),
    "mri_host_matmul_int8": (_I, [_P, _P, _SZ, _F, _P, _SZ, _P, _P]),
    "mri_host_matmul_int8_from_f32": (_I, [_P, _P, _SZ, _SZ, _P, _P]),
    "mri_host_matmul_q8_0_direct": (_I, [_P, _P, _SZ, _SZ, _P, _P]),
    "mri_host_matmul_q4_0_dequant": (_I, [_P, _P, _SZ, _SZ, _P, _P]),
    "mri_int8_path": (_I, [_P, _SZ, _SZ, _SZ]),
    "mri_int8_gemv_plan": (_I, [_P, _SZ, _SZ, _SZ, _P]),
    "mri_int8_gemm_plan": (_I, [_P, _SZ, _SZ, _SZ, _P]),
    "mri_comm_available": (_I, []),
    "mri_comm_unique_id": (_I, [_P]),
    "mri_comm_create": (_I, [_P, _P, _I, _I, _I, _PP]),
    "mri_comm_destroy": (_I, [_P]),
    "mri_comm_rank": (_I, [_P, ctypes.POINTER(_I), ctypes.POINTER(_I)]),
    "mri_comm_wait": (_I, [_P]),
    "mri_shard_rows": (_I, [_SZ, _I, _I, ctypes.POINTER(_SZ), ctypes.POINTER(_SZ)]),
    "mri_sharded_matmul_int8_from_f32": (_I, [_P, _P, _SZ, _SZ, _P, _SZ, _P]),
    "mri_qmatrix_from_gguf": (_I, [_P, _I, _P, _SZ, _SZ, _SZ, _PP]),
    "mri_qmatrix_download": (_I, [_P, _P, _P]),
    "mri_gguf_dequant": (_I, [_P, _I, _P, _SZ, _SZ, _P]),
    "mri_llama_create": (_I, [_P, _P, _PP]),
    "mri_llama_free": (_I, [_P]),
    "mri_llama_last_error": (ctypes.c_char_p, []),
    "mri_llama_set_rope": (_I, [_P, _P, _P]),
    "mri_llama_set_embedding": (_I, [_P, _P]),
    "mri_llama_set_norms": (_I, [_P, _P, _P, _P]),
    "mri_llama_set_layer": (_I, [_P, ctypes.c_uint32] + [_P] * 14),
    "mri_llama_set_output": (_I, [_P, _P, _P]),
    "mri_llama_load_tensor": (_I, [_P, _I, ctypes.c_uint32, _I, _P, _SZ, _SZ, _SZ]),
    "mri_llama_init_random": (_I, [_P, ctypes.c_uint64]),
    "mri_llama_forward": (_I, [_P, _P, _SZ, _P]),
    "mri_llama_forward_at": (_I, [_P, _P, _SZ, _SZ, _P]),
    "mri_llama_block_forward": (_I, [_P, ctypes.c_uint32, _P, _SZ, _SZ, _P]),
    "mri_llama_set_option": (_I, [_P, _I, _I]),
    "mri_llama_attention_fallbacks": (_I, [_P, ctypes.POINTER(_SZ)]),
    "mri_llama_forward_decode": (_I, [_P, ctypes.c_uint32, _SZ, _P]),
    "mri_llama_generate_greedy": (_I, [_P, _P, _SZ, _SZ, _P, _P, _P]),
    "mri_llama_launches_per_decode_step": (_I, [_P, ctypes.POINTER(_SZ)]),
    "mri_matmul_int8_from_f32_noalloc": (_I, [_P, _SZ, _SZ, _P, _P, _SZ, _P, _P]),
    "mri_noalloc_last_error": (ctypes.c_char_p, []),
    "mri_noalloc_check_status": (_I, [_P]),
}

_lock = threading.Lock()
_lib = None


def library_path():
    return _build.LIB


def load(build_if_missing=True):
    """Loads (building first when stale) the C-ABI library."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if build_if_missing:
            _build.build()
        if not os.path.exists(_build.LIB):
            raise ImportError(f"libmri_gpu.so not found at {_build.LIB}; run build.py")
        lib = ctypes.CDLL(_build.LIB)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.mri_abi_version() != 1:
            raise ImportError("libmri_gpu.so ABI version mismatch")
        _lib = lib
        return lib


def last_error():
    return load().mri_last_error().decode(errors="replace")
