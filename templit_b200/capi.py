"""ctypes bindings of the C ABIs in include/templit_cuda.h (kernel library)
and include/templit_gpt.h (GPT training step on cuda::Runtime).

The libraries are built in-tree by ``make -C templit_b200`` (or
``__graft_entry__.build()``) into ``templit_b200/_build``.  Loading fails
loudly when they are missing: there is no fallback implementation.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import (POINTER, Structure, c_char_p, c_double, c_float, c_int, c_int32,
                    c_size_t, c_uint8, c_uint32, c_uint64, c_void_p)

BUILD_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_build")

TL_MAX_RANK = 8
TL_GEMM_MAX_GROUPS = 4
TL_ATTN_BHTD = 0
TL_ATTN_BTHD = 1
TL_ATTN_FORWARD, TL_ATTN_BACKWARD_Q, TL_ATTN_PRODUCT_TN = range(3)
TL_GEMM_GROUP_NONE, TL_GEMM_GROUP_N, TL_GEMM_GROUP_K = 0, 1, 2
TL_GEMM_MAX_BATCH_RANK = 6
TL_OPT_CHUNK = 8192

# enums (include/templit_cuda.h)
TL_OK, TL_ERR_INVALID, TL_ERR_CUDA, TL_ERR_UNSUPPORTED, TL_ERR_RANGE = range(5)
TL_FLAG_INDEX_RANGE, TL_FLAG_TIMEOUT = 1, 2
TL_ADD, TL_SUB, TL_MUL, TL_DIV = range(4)
TL_SCALAR_ADD, TL_SCALAR_DIV, TL_SCALAR_POW = range(3)
TL_SIGMOID, TL_SQRT, TL_EXP, TL_GELU, TL_GELU_DERIVATIVE = range(5)
TL_REDUCE_SUM, TL_REDUCE_MAX = range(2)
TL_REDUCE_MAX_GROUPS = 4
TL_GEMM_TF32, TL_GEMM_FP32, TL_GEMM_3XTF32 = range(3)


class TlParamSlot(Structure):
    _fields_ = [("param", c_void_p), ("out", c_void_p), ("grad", c_void_p),
                ("m1", c_void_p), ("m2", c_void_p), ("count", c_uint64),
                ("chunk0", c_uint32), ("step", c_uint32)]


class TlGemmDesc(Structure):
    _fields_ = [("a", c_void_p), ("b", c_void_p), ("c", c_void_p),
                ("bias", c_void_p), ("gelu_out", c_void_p),
                ("m", c_uint32), ("n", c_uint32), ("k", c_uint32),
                ("trans_a", c_int32), ("trans_b", c_int32),
                ("precision", c_int32), ("beta", c_float),
                ("batch_rank", c_uint32),
                ("batch_shape", c_uint32 * TL_GEMM_MAX_BATCH_RANK),
                ("a_batch_stride", c_uint64 * TL_GEMM_MAX_BATCH_RANK),
                ("b_batch_stride", c_uint64 * TL_GEMM_MAX_BATCH_RANK),
                ("c_batch_stride", c_uint64 * TL_GEMM_MAX_BATCH_RANK),
                ("workspace", c_void_p), ("workspace_bytes", c_uint64),
                ("addend", c_void_p), ("lda", c_uint64), ("ldb", c_uint64), ("ldc", c_uint64),
                ("group_mode", c_int32), ("groups", c_uint32),
                ("a_group", c_void_p * TL_GEMM_MAX_GROUPS), ("b_group", c_void_p * TL_GEMM_MAX_GROUPS),
                ("c_group", c_void_p * TL_GEMM_MAX_GROUPS),
                ("bias_group", c_void_p * TL_GEMM_MAX_GROUPS), ("gelu_grad_x", c_void_p),
                ("c_heads", c_uint32), ("c_head_rows", c_uint32)]


class TlAttnView(Structure):
    _fields_ = [("p", c_void_p), ("batch_stride", c_uint64), ("head_stride", c_uint64),
                ("row_stride", c_uint64), ("transposed", c_int32), ("reserved", c_int32)]


class TlAttnDesc(Structure):
    _fields_ = [("pass", c_int32), ("B", c_uint32), ("T", c_uint32), ("H", c_uint32),
                ("D", c_uint32), ("q", TlAttnView), ("k", TlAttnView), ("v", TlAttnView),
                ("o", TlAttnView), ("d_o", TlAttnView), ("dq", TlAttnView), ("dk", TlAttnView),
                ("divisor", c_void_p), ("mask", c_void_p), ("p", c_void_p), ("ds", c_void_p),
                ("workspace", c_void_p), ("workspace_bytes", c_uint64),
                ("mask_flag", c_void_p)]


class TlFlashDesc(Structure):
    _fields_ = [("B", c_uint32), ("T", c_uint32), ("H", c_uint32), ("D", c_uint32),
                ("q", TlAttnView), ("k", TlAttnView), ("v", TlAttnView), ("o", TlAttnView),
                ("d_o", TlAttnView), ("dq", TlAttnView), ("dk", TlAttnView), ("dv", TlAttnView),
                ("divisor", c_void_p), ("mask", c_void_p), ("mask_flag", c_void_p),
                ("lse", c_void_p), ("delta", c_void_p)]


class TlgConfig(Structure):
    _fields_ = [("family", c_uint32), ("batch", c_uint32), ("seq", c_uint32),
                ("seed", c_uint32), ("init_std", c_float), ("lr", c_float),
                ("beta1", c_float), ("beta2", c_float), ("eps", c_float),
                ("weight_decay", c_float), ("clip", c_float),
                ("world", c_uint32), ("fusion", c_int32), ("graphs", c_int32),
                ("gemm_precision", c_int32), ("deferred_wait", c_int32),
                ("micro_batches", c_uint32), ("flash_attention", c_int32)]


U32P = POINTER(c_uint32)

# name -> (restype, argtypes) of every entry point of templit_cuda.h
CUDA_ABI = {
    "tl_version": (c_int, []),
    "tl_last_error": (c_char_p, []),
    "tl_device_init": (c_int, [c_int]),
    "tl_device_status": (c_int, [U32P, c_void_p]),
    "tl_device_status_enqueue": (c_int, [U32P, c_void_p]),
    "tl_malloc": (c_int, [POINTER(c_void_p), c_size_t]),
    "tl_free": (c_int, [c_void_p]),
    "tl_host_alloc": (c_int, [POINTER(c_void_p), c_size_t]),
    "tl_host_free": (c_int, [c_void_p]),
    "tl_stream_create": (c_int, [POINTER(c_void_p)]),
    "tl_stream_destroy": (c_int, [c_void_p]),
    "tl_stream_sync": (c_int, [c_void_p]),
    "tl_memcpy_h2d": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    "tl_memcpy_d2h": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    "tl_memcpy_d2d": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    "tl_fill_u32": (c_int, [c_void_p, c_uint32, c_size_t, c_void_p]),
    "tl_event_create": (c_int, [POINTER(c_void_p)]),
    "tl_event_destroy": (c_int, [c_void_p]),
    "tl_event_record": (c_int, [c_void_p, c_void_p]),
    "tl_event_elapsed_ms": (c_int, [POINTER(c_float), c_void_p, c_void_p]),
    "tl_event_query": (c_int, [c_void_p, POINTER(c_int)]),
    "tl_attention_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                 c_void_p, c_uint32, c_uint32, c_uint32, c_uint32, c_int32,
                                 c_int32, c_void_p, c_size_t, c_void_p]),
    "tl_attention_bwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                 c_void_p, c_void_p, c_void_p, c_uint32, c_uint32, c_uint32,
                                 c_uint32, c_int32, c_int32, c_void_p, c_size_t, c_void_p]),
    "tl_attention_workspace_size": (c_size_t, [c_uint32, c_uint32, c_uint32, c_uint32]),
    "tl_attention_fused_supported": (c_int, [c_void_p]),
    "tl_attention_fused": (c_int, [c_void_p, c_void_p]),
    "tl_flash_attention_supported": (c_int, [POINTER(TlFlashDesc)]),
    "tl_flash_attention_fwd": (c_int, [POINTER(TlFlashDesc), c_void_p]),
    "tl_flash_attention_bwd": (c_int, [POINTER(TlFlashDesc), c_void_p]),
    "tl_flash_attention_probs": (c_int, [POINTER(TlFlashDesc), c_void_p, c_void_p]),
    "tl_attention_mask_check": (c_int, [c_void_p, c_uint32, c_void_p, c_void_p]),
    "tl_check_wait_timeout": (c_int, [c_uint64, c_void_p, c_void_p]),
    "tl_graph_capture_begin": (c_int, [c_void_p]),
    "tl_graph_capture_end": (c_int, [c_void_p, POINTER(c_void_p)]),
    "tl_graph_launch": (c_int, [c_void_p, c_void_p]),
    "tl_graph_destroy": (c_int, [c_void_p]),
    "tl_kernel_launches": (c_uint64, []),
    "tl_binary": (c_int, [c_int, c_void_p, U32P, c_int, c_void_p, U32P, c_int,
                          c_void_p, U32P, c_int, c_void_p]),
    "tl_scalar": (c_int, [c_int, c_void_p, c_float, c_void_p, c_size_t, c_void_p]),
    "tl_unary": (c_int, [c_int, c_void_p, c_void_p, c_size_t, c_void_p]),
    "tl_gelu_backward": (c_int, [c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "tl_copy": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    "tl_reduce": (c_int, [c_int, c_void_p, U32P, c_int, c_void_p, U32P, c_int,
                          c_void_p, c_size_t, c_void_p]),
    "tl_reduce_workspace_size": (c_size_t, [U32P, c_int, U32P, c_int]),
    "tl_reduce_group": (c_int, [c_int, ctypes.c_uint32, c_void_p, U32P, c_int, c_void_p, U32P,
                                c_int, c_void_p, c_size_t, c_void_p]),
    "tl_reduce_group_workspace_size": (c_size_t, [ctypes.c_uint32, U32P, c_int, U32P, c_int]),
    "tl_reduce_noalloc": (c_int, [c_int, c_void_p, U32P, c_int, c_void_p, U32P, c_int,
                                  c_void_p]),
    "tl_reduce_noalloc_max_workspace": (c_size_t, []),
    "tl_argmax": (c_int, [c_void_p, c_size_t, c_void_p, c_void_p, c_size_t, c_void_p]),
    "tl_argmax_workspace_size": (c_size_t, [c_size_t]),
    "tl_transpose": (c_int, [c_void_p, U32P, c_int, c_int, c_int, c_void_p, c_void_p]),
    "tl_softmax_rows": (c_int, [c_void_p, c_void_p, c_uint32, c_uint32, c_void_p]),
    "tl_softmax_scaled_masked_rows": (c_int, [c_void_p, c_void_p, c_void_p, c_uint32,
                                              c_void_p, c_uint32, c_uint32, c_void_p]),
    "tl_softmax_backward_rows": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_uint32,
                                         c_uint32, c_void_p]),
    "tl_rms_rows": (c_int, [c_void_p, c_void_p, c_uint32, c_uint32, c_void_p]),
    "tl_rmsnorm_rows": (c_int, [c_void_p, c_void_p, c_void_p, c_uint32, c_uint32,
                                c_void_p]),
    "tl_rmsnorm_backward_rows": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                         c_uint32, c_uint32, c_void_p]),
    "tl_xent_rows": (c_int, [c_void_p, c_void_p, c_void_p, c_uint32, c_uint32, c_void_p]),
    "tl_xent_backward_rows": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_uint32,
                                      c_uint32, c_void_p]),
    "tl_embedding_gather": (c_int, [c_void_p, c_uint32, c_uint32, c_void_p, c_uint32,
                                    c_void_p, c_void_p]),
    "tl_embedding_scatter_add": (c_int, [c_void_p, c_void_p, c_uint32, c_uint32, c_void_p,
                                         c_void_p, c_uint32, c_void_p, c_size_t, c_void_p]),
    "tl_embedding_scatter_workspace_size": (c_size_t, [c_uint32, c_uint32, c_uint32]),
    "tl_grad_sqnorm_accumulate": (c_int, [c_void_p, c_size_t, c_void_p, c_void_p,
                                          c_size_t, c_void_p]),
    "tl_grad_sqnorm_workspace_size": (c_size_t, [c_size_t]),
    "tl_clip_gradient": (c_int, [c_void_p, c_void_p, c_float, c_void_p, c_size_t, c_void_p]),
    "tl_adamw": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                         c_void_p, c_void_p, c_void_p, c_float, c_uint32, c_size_t,
                         c_void_p]),
    "tl_multi_clip_adamw": (c_int, [c_void_p, c_uint32, c_uint32, c_void_p, c_float,
                                    c_void_p, c_void_p, c_void_p, c_void_p, c_float,
                                    c_void_p, c_size_t, c_void_p]),
    "tl_multi_clip_adamw_workspace_size": (c_size_t, [c_uint32]),
    "tl_multi_grad_flat": (c_int, [c_void_p, c_uint32, c_uint32, c_void_p, c_int, c_void_p]),
    "tl_gemm": (c_int, [POINTER(TlGemmDesc), c_void_p]),
    "tl_gemm_workspace_size": (c_size_t, [POINTER(TlGemmDesc)]),
    "tl_gemm_on_tensor_cores": (c_int, [POINTER(TlGemmDesc)]),
    "tl_gemm_counters": (None, [POINTER(c_uint64), POINTER(c_uint64), POINTER(c_uint64)]),
}

GPT_ABI = {
    "tlg_last_error": (c_char_p, []),
    "tlg_create": (c_int, [POINTER(TlgConfig), POINTER(c_void_p)]),
    "tlg_destroy": (c_int, [c_void_p]),
    "tlg_set_batch": (c_int, [c_void_p, U32P, U32P]),
    "tlg_train_step": (c_int, [c_void_p, POINTER(c_float)]),
    "tlg_forward": (c_int, [c_void_p, POINTER(c_float)]),
    "tlg_param_count": (c_int, [c_void_p, POINTER(c_uint64), POINTER(c_uint32)]),
    "tlg_get_params": (c_int, [c_void_p, POINTER(c_float), c_uint64]),
    "tlg_set_params": (c_int, [c_void_p, POINTER(c_float), c_uint64]),
    "tlg_stream": (c_void_p, [c_void_p]),
    "tlg_stats": (c_int, [c_void_p, POINTER(c_uint64)]),
    "tlg_nccl_unique_id": (c_int, [POINTER(c_uint8)]),
    "tlg_set_communicator": (c_int, [c_void_p, POINTER(c_uint8), c_int, c_int]),
    "tlg_profile": (c_int, [c_void_p, c_char_p, c_int]),
    "tlg_loader_create": (c_int, [c_char_p, c_double, c_int, c_uint32, c_uint32, c_uint32,
                                  POINTER(c_void_p)]),
    "tlg_loader_next": (c_int, [c_void_p, POINTER(U32P), POINTER(U32P)]),
    "tlg_loader_destroy": (c_int, [c_void_p]),
    "tlg_save": (c_int, [c_void_p, c_char_p, c_int]),
    "tlg_load": (c_int, [c_void_p, c_char_p, c_int]),
    "tlg_infer_create": (c_int, [POINTER(TlgConfig), POINTER(c_void_p)]),
    "tlg_infer_destroy": (c_int, [c_void_p]),
    "tlg_infer_param_count": (c_int, [c_void_p, POINTER(c_uint64)]),
    "tlg_infer_get_params": (c_int, [c_void_p, POINTER(c_float), c_uint64]),
    "tlg_infer_set_params": (c_int, [c_void_p, POINTER(c_float), c_uint64]),
    "tlg_infer_logits": (c_int, [c_void_p, U32P, POINTER(c_float)]),
    "tlg_infer_generate": (c_int, [c_void_p, U32P, c_uint32, c_uint32, c_uint32, c_uint32,
                                   c_float, c_uint32, U32P, c_uint32, U32P]),
    "tlg_mlp_train": (c_int, [POINTER(c_float), c_uint32, c_uint32, c_uint32, c_uint32,
                              POINTER(c_float), POINTER(c_float), POINTER(c_float),
                              POINTER(c_float), POINTER(c_float), c_float, c_float, c_int,
                              c_int, POINTER(c_float), POINTER(ctypes.c_double)]),
    "tlg_mlp_last_error": (c_char_p, []),
}

_libs: dict[str, ctypes.CDLL] = {}


def library_path(name: str) -> str:
    return os.path.join(BUILD_DIR, name)


def _load(name: str, abi: dict) -> ctypes.CDLL:
    if name in _libs:
        return _libs[name]
    path = library_path(name)
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is not built; run `make -C templit_b200` "
                           "(the CUDA backend has no fallback)")
    lib = ctypes.CDLL(path, mode=ctypes.RTLD_GLOBAL)
    for fn, (res, args) in abi.items():
        f = getattr(lib, fn)
        f.restype = res
        f.argtypes = args
    _libs[name] = lib
    return lib


def cuda_lib() -> ctypes.CDLL:
    return _load("libtemplit_cuda.so", CUDA_ABI)


def gpt_lib() -> ctypes.CDLL:
    cuda_lib()
    return _load("libtemplit_gpt.so", GPT_ABI)


class TlError(RuntimeError):
    pass


def check(rc: int, lib: ctypes.CDLL | None = None, what: str = "") -> None:
    if rc != 0:
        lib = lib or cuda_lib()
        msg = (lib.tlg_last_error() if hasattr(lib, "tlg_last_error")
               else lib.tl_last_error())
        raise TlError(f"{what} failed ({rc}): {msg.decode() if msg else ''}")


def shape_arr(shape) -> ctypes.Array:
    arr = (c_uint32 * max(1, len(shape)))()
    for i, s in enumerate(shape):
        arr[i] = int(s)
    return arr
