"""ctypes binding of libb200quant.so (C ABI declared in include/b200quant.h).

The library is the only compute path of this package: if it is missing or
cannot be loaded, every entry point raises -- there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / 'libb200quant.so'
HEADER = PKG.parent / 'include' / 'b200quant.h'

B200Q_OK, B200Q_EINVAL, B200Q_ECUDA, B200Q_ETIMEOUT, B200Q_ENODEV, B200Q_EINDEX = 0, -1, -2, -3, -4, -5

_u8p = ctypes.POINTER(ctypes.c_uint8)
_f32p = ctypes.POINTER(ctypes.c_float)
_vp = ctypes.c_void_p
_u32 = ctypes.c_uint
_i, _ll, _sz = ctypes.c_int, ctypes.c_longlong, ctypes.c_size_t

# name -> (restype, argtypes); every function declared in include/b200quant.h
SIGNATURES = {
    'localai_q8_0_matvec': (None, [_u8p, _f32p, _f32p, _i, _i, _i]),
    'localai_q4_0_matvec': (None, [_u8p, _f32p, _f32p, _i, _i, _i]),
    'localai_q4k_matvec': (None, [_u8p, _f32p, _f32p, _i, _i, _i]),
    'localai_q5k_matvec': (None, [_u8p, _f32p, _f32p, _i, _i, _i]),
    'localai_q6k_matvec': (None, [_u8p, _f32p, _f32p, _i, _i, _i]),
    'localai_q8_0_matmul': (None, [_u8p, _f32p, _f32p, _i, _i, _i, _i]),
    'localai_q4_0_matmul': (None, [_u8p, _f32p, _f32p, _i, _i, _i, _i]),
    'localai_q4k_matmul': (None, [_u8p, _f32p, _f32p, _i, _i, _i, _i]),
    'localai_q5k_matmul': (None, [_u8p, _f32p, _f32p, _i, _i, _i, _i]),
    'localai_q6k_matmul': (None, [_u8p, _f32p, _f32p, _i, _i, _i, _i]),
    'b200q_matmul_tensor_core_min_tokens': (_i, [_i]),
    'b200q_last_status': (_i, []),
    'b200q_last_error': (ctypes.c_char_p, []),
    'b200q_init': (_i, [_i]),
    'b200q_register_host': (_i, [_vp, _sz]),
    'b200q_unregister_host': (_i, [_vp]),
    'b200q_registry_clear': (_i, []),
    'b200q_registered_device_ptr': (_vp, [_vp]),
    'b200q_dequant_f32_dev': (_i, [_i, _vp, _vp, _ll, _vp]),
    'b200q_dequant_bf16_dev': (_i, [_i, _vp, _vp, _ll, _vp]),
    'b200q_gemv_dev': (_i, [_i, _vp, _vp, _vp, _i, _i, _i, _ll, _ll, _vp]),
    'b200q_gemm_q4k_dev': (_i, [_vp, _ll, _i, _vp, _i, _i, _i, _i, _vp, _vp, _i, _vp, _i, _ll, _vp, _vp, _ll, _i, _vp]),
    'b200q_zaya_router_prep_dev': (_i, [_vp, _vp, _vp, _vp, _i, _i, ctypes.c_float, _vp, _vp, _vp]),
    'b200q_gelu_dev': (_i, [_vp, _ll, _vp]),
    'b200q_copy_rows_range_dev': (_i, [_vp, _vp, _vp, _i, _i, _i, _vp]),
    'b200q_silu_mul_dev': (_i, [_vp, _i, _i, _vp, _ll, _vp]),
    'b200q_gemv_grouped_max_tokens': (_i, [_i, _i]),
    'b200q_gemv_grouped_dev': (_i, [_i, _vp, _ll, _ll, _i, _vp, _vp, _vp, _ll, _i, _i, _i, _i, _i, _vp]),
    'b200q_moe_gather_f32_dev': (_i, [_vp, _i, _vp, _i, _i, _vp, _vp]),
    'b200q_moe_gather_bf16_dev': (_i, [_vp, _i, _vp, _i, _i, _vp, _vp]),
    'b200q_moe_scatter_bf16_dev': (_i, [_vp, _i, _vp, _i, _i, _i, _vp, _vp]),
    'b200q_gemm_dev': (_i, [_i, _vp, _ll, _i, _vp, _ll, _i, _i, _i, _i, _vp, _vp, _i, _vp, _i, _ll, _vp, _vp, _ll,
                            _i, _vp]),
    'b200q_moe_router_dev': (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    'b200q_moe_topk_dev': (_i, [_vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp]),
    'b200q_moe_num_blocks': (_i, [_i]),
    'b200q_moe_route_workspace_bytes': (_sz, [_i, _i, _i]),
    'b200q_moe_route_dev': (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _sz, _vp]),
    'b200q_moe_route_bf16_dev': (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _sz, _vp, _vp]),
    'b200q_moe_dispatch_dev': (_i, [_vp, _vp, _i, _i, _i, _vp, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    'b200q_moe_dispatch_noalloc_dev': (_i, [_vp, _vp, _i, _i, _i, _vp, _i, _vp, _vp, _vp, _vp, _vp, _vp]),
    'b200q_moe_combine_dev': (_i, [_vp, _i, _vp, _vp, _i, _i, _i, _vp, _vp]),
    'b200q_check_device_error': (_i, []),
    'b200q_gemv_tuning': (None, [_i, _i, _i, _i]),
    'b200q_gemv_mma_tuning': (None, [_i, _i, _i, _i]),
    'b200q_gemm_pair_mode': (_i, [_i]),
    'b200q_launch_count': (_ll, []),
    'b200q_dequant_row_dev': (_i, [_i, _vp, _ll, _i, _vp, _i, _i, _vp, _vp]),
    'b200q_add_rmsnorm_dev': (_i, [_vp, _vp, _vp, _i, _i, ctypes.c_float, _vp, _vp, _vp]),
    'b200q_rope_kv_dev': (_i, [_vp, _i, _i, _i, _i, _i, ctypes.c_float, _vp, _vp, _vp, _i, _vp]),
    'b200q_rope_kv_ex_dev': (_i, [_vp, _i, _i, _i, _i, _i, ctypes.c_float, _vp, _i, _vp, _vp, _vp, _i, _vp]),
    'b200q_qkv_bias_norm_dev': (_i, [_vp, _i, _i, _i, _i, _vp, _vp, _vp, ctypes.c_float, _vp]),
    'b200q_attn_prefill_dev': (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp]),
    'b200q_attn_prefill_ex_dev': (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp, _vp]),
    'b200q_attn_prefill_tc_scratch_bytes': (_sz, [_i, _i, _i, _i, _i]),
    'b200q_attn_prefill_tc_dev': (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _sz, _vp, _vp]),
    'b200q_attn_decode_scratch_floats': (_sz, [_i, _i, _i]),
    'b200q_attn_decode_dev': (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp]),
    'b200q_attn_decode_ex_dev': (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp, _vp]),
    'b200q_argmax_dev': (_i, [_vp, _i, _vp, _vp, _vp, _i, _vp, _vp]),
    'b200q_ep_create': (_i, [_i, _i, _i, _i, _ll, _ll, ctypes.POINTER(_vp)]),
    'b200q_ep_handle_bytes': (_sz, []),
    'b200q_ep_set_wait_limit_ns': (None, [ctypes.c_ulonglong]),
    'b200q_ep_handle': (_i, [_vp, _vp]),
    'b200q_ep_open': (_i, [_vp, _vp]),
    'b200q_ep_destroy': (_i, [_vp]),
    'b200q_ep_recv_rows': (_vp, [_vp]),
    'b200q_ep_return_rows': (_vp, [_vp]),
    'b200q_ep_group_offsets': (_vp, [_vp]),
    'b200q_ep_exchange_counts_dev': (_i, [_vp, _vp, _u32, _vp]),
    'b200q_ep_send_rows_dev': (_i, [_vp, _vp, _i, _vp, _vp, _i, _u32, _vp]),
    'b200q_ep_send_rows_bf16_dev': (_i, [_vp, _vp, _i, _vp, _vp, _i, _u32, _vp]),
    'b200q_ep_experts_dev': (_i, [_vp, _i, _vp, _ll, _vp, _ll, _i, _vp, _u32, _i, _vp]),
    'b200q_ep_dispatch_experts_dev': (_i, [_vp, _i, _vp, _ll, _vp, _ll, _i, _vp, _vp, _i, _vp, _vp, _i, _u32, _i,
                                           _vp]),
    'b200q_ep_combine_dev': (_i, [_vp, _vp, _vp, _i, _i, _vp, _u32, _vp]),
}

_LIB = None


class B200QError(RuntimeError):
    """A libb200quant call failed (message from b200q_last_error)."""


def header_functions() -> list[str]:
    """Names of every function declared in include/b200quant.h."""
    text = HEADER.read_text()
    text = re.sub(r'/\*.*?\*/', '', text, flags=re.S)
    return re.findall(r'\b((?:localai|b200q)_\w+)\s*\(', text)


def load() -> ctypes.CDLL:
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise B200QError(f'{LIB_PATH.name} is not built; run `python -m localai_b200.build`')
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


def check(status: int | None = None) -> None:
    """Raise B200QError if ``status`` (or the library's last status) is an error."""
    lib = load()
    code = lib.b200q_last_status() if status is None else status
    if code != B200Q_OK:
        msg = lib.b200q_last_error().decode(errors='replace')
        raise B200QError(f'libb200quant error {code}: {msg}')


def launch_count() -> int:
    return int(load().b200q_launch_count())
