"""ctypes binding of ``libs8b.so`` (the C ABI declared in ``include/s8b.h``).

There is no fallback: if the library is missing, or a tensor handed to it is not on a CUDA
device, the call raises. Status codes other than 0 become ``S8BError``.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libs8b.so"

S8B_BF16, S8B_FP16 = 0, 1
CODEC = {"fp16": 0, "int8": 1, "int8-had": 2, "int4": 3, "int4-had": 4, "nf4": 5}
ERR_TIMEOUT = -6

_vp, _i, _f, _sz, _u32, _u64 = C.c_void_p, C.c_int, C.c_float, C.c_size_t, C.c_uint32, C.c_uint64

# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple] = {
    "s8b_strerror": (C.c_char_p, [_i]),
    "s8b_version": (_i, []),
    "s8b_last_cuda_error": (_i, []),
    "s8b_launch_count": (C.c_ulonglong, []),
    "s8b_quant_rows": (_i, [_vp, _i, _vp, _vp, _i, _i, _vp]),
    "s8b_rmsnorm_quant": (_i, [_vp, _vp, _vp, _vp, _f, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "s8b_gemm_w8a8": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp]),
    "s8b_silu_mul_quant": (_i, [_vp, _i, _i, _vp, _vp, _vp, _i, _vp]),
    "s8b_rmsnorm_quant_split": (_i, [_vp, _i, _vp, _vp, _vp, _vp, _vp, _f, _vp, _vp, _vp, _i,
                                     _i, _i, _vp]),
    "s8b_silu_mul_quant_split": (_i, [_vp, _i, _vp, _vp, _i, _i, _vp, _vp, _vp, _i, _vp]),
    "s8b_qkv_post_split": (_i, [_vp, _i, _vp, _vp, _vp, _vp, _vp, _i, _vp, _vp, _f, _i, _i, _i,
                                _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i,
                                _vp]),
    "s8b_gemm_tc_workspace_size": (_sz, [_i, _i]),
    "s8b_gemm_tc_split_count": (_i, [_i, _i, _i]),
    "s8b_gemm_w8a8_tc": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _sz, _vp]),
    "s8b_tc_packed_bytes": (_sz, [_i, _i]),
    "s8b_pack_weights_tc": (_i, [_vp, _i, _i, _vp, _vp]),
    "s8b_gemm_w8a8_tc_packed": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _sz,
                                     _vp]),
    "s8b_qkv_post": (_i, [_vp, _vp, _vp, _vp, _i, _vp, _vp, _f, _i, _i, _i, _i, _vp, _vp, _vp,
                          _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "s8b_kv_write_paged": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp]),
    "s8b_paged_decode_workspace_size": (_sz, [_i, _i, _i, _i]),
    "s8b_paged_decode_status_offset": (_sz, [_i, _i]),
    "s8b_set_attention_impl": (_i, [_i]),
    "s8b_paged_decode_q8": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i,
                                 _i, _i, _i, _i, _i, _f, _vp, _sz, _i, _vp]),
    "s8b_paged_decode_q8_step": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                      _i, _i, _i, _i, _i, _i, _i, _f, _vp, _sz, _i, _vp]),
    "s8b_paged_prefill_block_rows": (_i, [_i, _i]),
    "s8b_paged_prefill_q8": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp, _vp, _vp,
                                  _i, _i, _i, _i, _i, _i, _i, _f, _vp, _sz, _i, _vp]),
    "s8b_paged_decode_q8_noalloc": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                         _i, _i, _i, _i, _i, _i, _i, _f, _i, _vp]),
    "s8b_paged_decode_noalloc_status": (_i, [_vp, C.c_int32]),
    "s8b_paged_decode_ref_workspace_size": (_sz, [_i, _i, _i, _i]),
    "s8b_paged_decode": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i,
                              _i, _f, _vp, _sz, _i, _vp]),
    "s8b_embed": (_i, [_vp, _vp, _i, _i, _vp, _i, _vp]),
    "s8b_argmax": (_i, [_vp, _i, _i, _vp, _i, _vp]),
    "s8b_exp_f32": (_i, [_vp, _vp, C.c_longlong, _vp]),
    "s8b_codec_payload_bytes": (_sz, [_i, _i, _i, _i]),
    "s8b_codec_scale_count": (_sz, [_i, _i, _i]),
    "s8b_codec_encode": (_i, [_vp, _vp, _i, _i, _i, _i, _vp, _vp, _i, _vp]),
    "s8b_codec_decode": (_i, [_vp, _vp, _i, _i, _i, _i, _vp, _vp, _i, _vp]),
    "s8b_codec_encode_split": (_i, [_vp, _i, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp, _i, _vp]),
    "s8b_rmsnorm_quant_codec": (_i, [_vp, _vp, _i, _vp, _vp, _f, _vp, _vp, _i, _i, _i, _vp]),
    "s8b_flag_set": (_i, [_vp, _vp, _u32, _vp]),
    "s8b_flag_wait": (_i, [_vp, _vp, _u32, _u64, _vp, _vp]),
    "s8b_counter_add": (_i, [_vp, _u32, _vp]),
    "s8b_peer_put_flag": (_i, [_vp, _vp, _vp, _i, _vp, _vp, _u32, _vp]),
    "s8b_flag_status": (_i, [_vp]),
    "s8b_advance": (_i, [_vp, _vp, _i, _i, _vp]),
    "s8b_enable_peer_access": (_i, [_i, _i]),
    "s8b_ipc_handle_size": (_i, []),
    "s8b_ipc_alloc": (_i, [_sz, _vp, _vp]),
    "s8b_ipc_free": (_i, [_vp]),
    "s8b_ipc_open": (_i, [_vp, _vp]),
    "s8b_ipc_close": (_i, [_vp]),
    "s8b_memcpy_async": (_i, [_vp, _vp, _sz, _vp]),
    "s8b_moe_route": (_i, [_vp, _i, _vp, _i, _i, _i, _i, _i, _f, _vp, _vp, _vp, _vp, _vp, _vp,
                           _vp]),
    "s8b_moe_gemm_grouped": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp]),
    "s8b_moe_combine": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "s8b_moe_gemm_grouped_tc": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _i,
                                     _vp]),
    "s8b_moe_gather_rows": (_i, [_vp, _vp, _vp, _i, _i, _vp, _vp, _vp]),
    "s8b_rans_encoded_capacity": (_sz, [_sz, _i]),
    "s8b_rans_stream_offset": (_sz, [_sz, _i, _i]),
    "s8b_rans_histogram": (_i, [_vp, _sz, _vp, _vp]),
    "s8b_rans_encode": (_i, [_vp, _sz, _vp, _i, _vp, _sz, _vp, _vp]),
    "s8b_rans_decode": (_i, [_vp, _vp, _i, _vp, _sz, _vp, _vp, _vp]),
    "s8b_stage_step": (_i, [_vp, _vp]),
    "s8b_stage_desc_size": (_sz, []),
    "s8b_layer_desc_size": (_sz, []),
    "s8b_sample_workspace_size": (_sz, [_i, _i]),
    "s8b_sample": (_i, [_vp, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp, _vp, _sz,
                        _vp, _vp]),
}


class S8BError(RuntimeError):
    def __init__(self, name: str, code: int, detail: str = ""):
        self.code = code
        super().__init__(f"{name} failed: {code} ({strerror(code)}){detail}")


_LIB: C.CDLL | None = None


def load() -> C.CDLL:
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH} is not built; run `python -m superl8_serve_b200.csrc.build` "
            "(there is no CPU fallback for the s8b kernels)")
    lib = C.CDLL(os.fspath(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


def strerror(code: int) -> str:
    return load().s8b_strerror(code).decode()


def call(name: str, *args) -> int:
    fn = getattr(load(), name)
    rc = fn(*args)
    if rc != 0:
        detail = ""
        if rc == -4:
            detail = f"; cudaError {load().s8b_last_cuda_error()}"
        raise S8BError(name, rc, detail)
    return rc


def ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise RuntimeError("s8b kernels take CUDA tensors only (no CPU fallback)")
    if not t.is_contiguous():
        raise RuntimeError("s8b kernels take contiguous tensors")
    return t.data_ptr()


def stream(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.bfloat16:
        return S8B_BF16
    if dt == torch.float16:
        return S8B_FP16
    raise RuntimeError(f"s8b activation dtype must be bf16 or fp16, got {dt}")
