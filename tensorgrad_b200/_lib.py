"""ctypes binding of ``libtgb200.so`` (declared in ``include/tgb200.h``).

The library must exist (``python -m tensorgrad_b200._build``) and a CUDA device must be
visible for any compute call: there is no CPU fallback, and importing an op module on a
machine without the library raises at the first call, loudly.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_double, c_int, c_int64, c_size_t, c_uint, c_void_p

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libtgb200.so")

F32, F64 = 0, 1
ADD, SUB, MUL, DIV, POW, EQ = 0, 1, 2, 3, 4, 5
(NEG, EXP, LOG, SQRT, TANH, SIGMOID, RELU, SQUARE, FILL, POWS, ABS, FINITE_OR_ZERO,
 LOG1P) = range(13)

_STATUS_ERRORS: dict[int, type[Exception]] = {
    1: ValueError,
    2: RuntimeError,
    3: NotImplementedError,
    4: IndexError,
    5: TimeoutError,
    6: MemoryError,
    7: RuntimeError,
}


class AttnShape(ctypes.Structure):
    """``tg_attn_shape``: (B, H, T, D) views through element strides."""

    _fields_ = [(name, c_int64) for name in (
        "batch", "heads", "tq", "tk", "head_dim",
        "q_sb", "q_sh", "q_st", "k_sb", "k_sh", "k_st",
        "v_sb", "v_sh", "v_st", "o_sb", "o_sh", "o_st",
    )] + [("causal", c_int)]


class ConvShape(ctypes.Structure):
    """``tg_conv_shape``: input (n, c, h, w), filters (c_out, kh, kw), stride, padding and
    the output size (oh, ow)."""

    _fields_ = [(name, c_int64) for name in (
        "n", "c", "h", "w", "c_out", "kh", "kw", "sh", "sw", "ph", "pw", "oh", "ow",
    )]


vp, i64, dbl, u32, sz = c_void_p, c_int64, c_double, c_uint, c_size_t
pi64 = POINTER(c_int64)
pint = POINTER(c_int)
pvp = POINTER(c_void_p)

#: name -> (restype, argtypes); every symbol of include/tgb200.h.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "tg_version": (c_int, []),
    "tg_status_string": (c_char_p, [c_int]),
    "tg_last_error": (c_int, [c_char_p, sz]),
    "tg_device_info": (c_int, [c_int, pint, pint, pint]),
    "tg_memcpy_h2d": (c_int, [vp, vp, sz, vp]),
    "tg_memcpy_d2h": (c_int, [vp, vp, sz, vp]),
    "tg_memcpy_d2d": (c_int, [vp, vp, sz, vp]),
    "tg_memset_zero": (c_int, [vp, sz, vp]),
    "tg_stream_synchronize": (c_int, [vp]),
    "tg_malloc": (c_int, [POINTER(c_void_p), sz, vp]),
    "tg_free": (c_int, [vp, vp]),
    "tg_pool_stats": (c_int, [c_int, POINTER(ctypes.c_uint64), POINTER(ctypes.c_uint64)]),
    "tg_pool_peak": (c_int, [c_int, c_int, POINTER(ctypes.c_uint64)]),
    "tg_host_alloc": (c_int, [POINTER(c_void_p), sz]),
    "tg_host_free": (c_int, [vp]),
    "tg_set_device": (c_int, [c_int]),
    "tg_get_device": (c_int, [pint]),
    "tg_device_count": (c_int, [pint]),
    "tg_event_create": (c_int, [POINTER(c_void_p)]),
    "tg_event_record": (c_int, [vp, vp]),
    "tg_event_query": (c_int, [vp]),
    "tg_event_destroy": (c_int, [vp]),
    "tg_comm_load": (c_int, [c_char_p]),
    "tg_comm_nccl_version": (c_int, [pint]),
    "tg_comm_unique_id": (c_int, [vp, sz]),
    "tg_comm_init": (c_int, [c_int, c_int, vp, dbl, POINTER(c_void_p)]),
    "tg_comm_all_reduce": (c_int, [vp, vp, sz, c_int, c_int, vp, dbl]),
    "tg_comm_join": (c_int, [vp, vp]),
    "tg_comm_wait": (c_int, [vp, dbl]),
    "tg_comm_abort": (c_int, [vp]),
    "tg_comm_destroy": (c_int, [vp, dbl]),
    "tg_gemm": (c_int, [c_int, c_int, c_int, i64, i64, i64, dbl, vp, i64, vp, i64, dbl, vp, i64,
                        vp, vp]),
    "tg_gemm_simt": (c_int, [c_int, c_int, c_int, i64, i64, i64, dbl, vp, i64, vp, i64, dbl, vp,
                             i64, vp, vp]),
    "tg_gemm_tc_status": (c_int, [c_int]),
    "tg_attention_tc_status": (c_int, [c_int]),
    "tg_attention_set_wait_test": (c_int, [i64, c_int]),
    "tg_test_exp_fma": (c_int, [i64, vp, vp, vp]),
    "tg_set_matmul_precision": (c_int, [c_int]),
    "tg_gemm_profile": (c_int, [c_int]),
    "tg_gemm_profile_read": (c_int, [POINTER(c_double), POINTER(c_int64), POINTER(c_double)]),
    "tg_launch_count": (ctypes.c_uint64, []),
    "tg_gemm_fallback_count": (ctypes.c_uint64, []),
    "tg_gemm_batched": (c_int, [c_int, c_int, c_int, i64, i64, i64, dbl, vp, i64, i64, vp, i64,
                                i64, dbl, vp, i64, i64, i64, vp]),
    "tg_linear_forward_scratch_bytes": (sz, [c_int, i64, i64, i64]),
    "tg_linear_forward": (c_int, [c_int, vp, vp, vp, vp, i64, i64, i64, vp, vp]),
    "tg_linear_backward_scratch_bytes": (sz, [c_int, i64, i64, i64, u32]),
    "tg_linear_backward": (c_int, [c_int, vp, vp, vp, vp, vp, vp, i64, i64, i64, u32, dbl, vp,
                                   vp]),
    "tg_colsum_scratch_bytes": (sz, [c_int, i64, i64]),
    "tg_colsum": (c_int, [c_int, vp, vp, i64, i64, c_int, vp, vp]),
    "tg_reduce_sum": (c_int, [c_int, c_int, pi64, pint, vp, vp, vp]),
    "tg_reduce_extremum": (c_int, [c_int, c_int, c_int, pi64, pint, vp, vp, vp]),
    "tg_reduce_truth": (c_int, [c_int, c_int, c_int, pi64, pint, vp, vp, vp]),
    "tg_argmax": (c_int, [c_int, c_int, pi64, pint, vp, vp, vp]),
    "tg_compare": (c_int, [c_int, c_int, c_int, pi64, vp, pi64, vp, pi64, vp, vp]),
    "tg_where": (c_int, [c_int, c_int, c_int, pi64, vp, pi64, vp, pi64, vp, pi64, vp, vp]),
    "tg_sum_all_scratch_bytes": (sz, []),
    "tg_sum_all": (c_int, [c_int, vp, vp, i64, vp, vp]),
    "tg_binary": (c_int, [c_int, c_int, c_int, pi64, vp, pi64, vp, pi64, vp, vp]),
    "tg_axpby": (c_int, [c_int, i64, dbl, vp, dbl, vp, vp, vp]),
    "tg_scale_by_device_scalar": (c_int, [c_int, i64, vp, vp, dbl, vp, vp]),
    "tg_unary": (c_int, [c_int, c_int, i64, vp, dbl, vp, vp]),
    "tg_cast": (c_int, [c_int, c_int, i64, vp, vp, vp]),
    "tg_strided_copy": (c_int, [c_int, c_int, pi64, vp, pi64, vp, pi64, vp]),
    "tg_gelu_forward": (c_int, [c_int, i64, vp, vp, vp]),
    "tg_gelu_backward": (c_int, [c_int, i64, vp, vp, vp, vp]),
    "tg_relu_backward": (c_int, [c_int, i64, vp, vp, vp, vp]),
    "tg_unary_backward": (c_int, [c_int, c_int, i64, vp, vp, vp, dbl, vp, vp]),
    "tg_dropout_pcg64": (c_int, [c_int, i64, vp, vp, POINTER(ctypes.c_uint64), i64, ctypes.c_uint32,
                                 dbl, vp]),
    "tg_layer_norm_forward": (c_int, [c_int, vp, vp, vp, vp, vp, vp, i64, i64, dbl, vp]),
    "tg_layer_norm_scratch_bytes": (sz, [c_int, i64, i64]),
    "tg_layer_norm_backward": (c_int, [c_int, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, u32, vp,
                                       vp]),
    "tg_layer_norm_backward_noalloc": (c_int, [c_int, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64,
                                               u32, vp]),
    "tg_embedding_forward": (c_int, [c_int, vp, vp, vp, i64, i64, i64, vp, vp]),
    "tg_embedding_backward": (c_int, [c_int, vp, vp, vp, vp, i64, vp, i64, i64, c_int, vp]),
    "tg_embedding_sort_scratch_bytes": (sz, [i64, i64]),
    "tg_embedding_sort": (c_int, [vp, i64, i64, vp, vp, vp, sz, vp]),
    "tg_embedding_backward_sorted": (c_int, [c_int, vp, vp, i64, vp, i64, i64, c_int, vp]),
    "tg_cross_entropy_forward": (c_int, [c_int, vp, vp, vp, vp, vp, i64, i64, i64, c_int, vp, vp,
                                         vp]),
    "tg_cross_entropy_backward": (c_int, [c_int, vp, vp, vp, vp, vp, vp, i64, i64, i64, c_int,
                                          vp]),
    "tg_attention_forward_scratch_bytes": (sz, [c_int, POINTER(AttnShape)]),
    "tg_attention_forward": (c_int, [c_int, POINTER(AttnShape), vp, vp, vp, vp, vp, vp, vp]),
    "tg_attention_backward_scratch_bytes": (sz, [c_int, POINTER(AttnShape)]),
    "tg_attention_backward": (c_int, [c_int, POINTER(AttnShape), vp, vp, vp, vp, vp, vp, vp, vp,
                                      vp, vp, vp]),
    "tg_attention_dropout_scratch_bytes": (sz, [c_int, POINTER(AttnShape)]),
    "tg_attention_forward_dropout": (c_int, [c_int, POINTER(AttnShape), vp, vp, vp, vp, vp,
                                             POINTER(ctypes.c_uint64), ctypes.c_uint32, dbl, vp,
                                             vp]),
    "tg_attention_backward_dropout": (c_int, [c_int, POINTER(AttnShape), vp, vp, vp, vp, vp, vp,
                                              vp, POINTER(ctypes.c_uint64), ctypes.c_uint32, dbl,
                                              vp, vp]),
    "tg_conv2d_cols_shape": (c_int, [POINTER(ConvShape), pi64, pi64]),
    "tg_conv2d_forward_scratch_bytes": (sz, [c_int, POINTER(ConvShape)]),
    "tg_conv2d_forward": (c_int, [c_int, POINTER(ConvShape), vp, vp, vp, vp, vp, vp, vp]),
    "tg_conv2d_im2col": (c_int, [c_int, POINTER(ConvShape), vp, vp, vp]),
    "tg_conv2d_backward_scratch_bytes": (sz, [c_int, POINTER(ConvShape), c_int]),
    "tg_conv2d_backward": (c_int, [c_int, POINTER(ConvShape), vp, vp, vp, vp, vp, vp, vp, vp]),
    "tg_batch_norm_scratch_bytes": (sz, [c_int, i64, i64, i64]),
    "tg_batch_norm_forward": (c_int, [c_int, i64, i64, i64, vp, vp, vp, vp, vp, vp, vp, vp, dbl,
                                      dbl, vp, vp]),
    "tg_batch_norm_backward": (c_int, [c_int, i64, i64, i64, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                                       vp]),
    "tg_max_pool2d_forward": (c_int, [c_int, POINTER(ConvShape), vp, vp, vp, vp]),
    "tg_max_pool2d_backward": (c_int, [c_int, POINTER(ConvShape), vp, vp, vp, vp]),
    "tg_max_pool2d_gather": (c_int, [c_int, POINTER(ConvShape), vp, vp, vp, vp]),
    "tg_lstm_forward_scratch_bytes": (sz, [c_int, i64, i64, i64, i64]),
    "tg_lstm_forward": (c_int, [c_int, i64, i64, i64, i64] + [vp] * 12),
    "tg_lstm_backward_scratch_bytes": (sz, [c_int, i64, i64, i64, i64]),
    "tg_lstm_backward": (c_int, [c_int, i64, i64, i64, i64] + [vp] * 18),
    "tg_gru_forward_scratch_bytes": (sz, [c_int, i64, i64, i64, i64]),
    "tg_gru_forward": (c_int, [c_int, i64, i64, i64, i64] + [vp] * 11),
    "tg_gru_backward_scratch_bytes": (sz, [c_int, i64, i64, i64, i64]),
    "tg_gru_backward": (c_int, [c_int, i64, i64, i64, i64] + [vp] * 16),
    "tg_rnn_forward_scratch_bytes": (sz, [c_int, i64, i64, i64, i64]),
    "tg_rnn_forward": (c_int, [c_int, c_int, i64, i64, i64, i64] + [vp] * 9),
    "tg_rnn_backward_scratch_bytes": (sz, [c_int, i64, i64, i64, i64]),
    "tg_rnn_backward": (c_int, [c_int, c_int, i64, i64, i64, i64] + [vp] * 14),
    "tg_sumsq_scratch_bytes": (sz, [c_int]),
    "tg_sumsq_multi": (c_int, [c_int, c_int, pvp, pi64, vp, vp, vp]),
    "tg_clip_scale_multi": (c_int, [c_int, c_int, pvp, pi64, vp, dbl, dbl, vp, vp]),
    "tg_adam_update": (c_int, [c_int, i64, vp, vp, vp, vp, dbl, dbl, dbl, dbl, dbl, i64, c_int,
                               vp]),
    "tg_adam_update_clipped": (c_int, [c_int, i64, vp, vp, vp, vp, dbl, dbl, dbl, dbl, dbl, i64,
                                       c_int, vp, dbl, dbl, vp]),
    "tg_adam_multi_scratch_bytes": (sz, [c_int]),
    "tg_adam_update_multi": (c_int, [c_int, c_int, pvp, pvp, pvp, pvp, pi64, pi64, dbl, dbl, dbl,
                                     dbl, dbl, c_int, vp, vp]),
}


class _Lib:
    """Lazily loaded library handle; attribute access returns the bound C function."""

    def __init__(self) -> None:
        self._dll: ctypes.CDLL | None = None

    def load(self) -> ctypes.CDLL:
        if self._dll is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build the CUDA kernels first "
                    "(python -m tensorgrad_b200._build); there is no CPU fallback"
                )
            dll = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(dll, name)
                fn.restype = res
                fn.argtypes = args
            self._dll = dll
        return self._dll

    def __getattr__(self, name: str):  # noqa: ANN204
        fn = getattr(self.load(), name)
        setattr(self, name, fn)
        return fn


lib = _Lib()


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    lib.tg_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(status: int, what: str = "") -> None:
    """Raise the exception type that the reference raises for this kind of failure."""
    if status:
        exc = _STATUS_ERRORS.get(status, RuntimeError)
        detail = last_error()
        raise exc(f"{what}: {detail}" if what else detail)


def int64_array(values: object) -> ctypes.Array:
    vals = list(values)  # type: ignore[call-overload]
    return (c_int64 * len(vals))(*vals)


def int_array(values: object) -> ctypes.Array:
    vals = list(values)  # type: ignore[call-overload]
    return (c_int * len(vals))(*vals)


def ptr_array(values: object) -> ctypes.Array:
    vals = list(values)  # type: ignore[call-overload]
    return (c_void_p * len(vals))(*vals)
