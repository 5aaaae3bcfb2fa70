"""ctypes binding of the C ABI declared in ``include/unblend_b200.h``.

The shared library is built in-tree (``python -m unblend_b200.build``). There is
no fallback: if the library is missing or a launcher returns an error, the
call raises. Launch errors carry the CUDA error text; an out-of-memory code is
reported with the words "CUDA out of memory" so ``apply_model``'s OOM backoff
(unblend/apply.py:32-53) still recognises it.
"""

from __future__ import annotations

import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_lib", "libunblend_b200.so")
ERR_INVALID = 1000
ERR_TOO_LARGE = 1001
NOALLOC_MAX_BATCH = 4096

c_int = ctypes.c_int
c_ll = ctypes.c_longlong
c_float = ctypes.c_float
c_double = ctypes.c_double
c_void_p = ctypes.c_void_p

ACT_NONE, ACT_GELU, ACT_GLU, ACT_TANH, ACT_SWISH = 0, 1, 2, 3, 4
PRO_NONE, PRO_GN_GELU, PRO_ADD = 0, 1, 2
GEMM_MAX_GROUPS = 64


class ConvParams(ctypes.Structure):
    """Mirror of ``UnblendConvParams``."""

    _fields_ = [
        ("batch", c_int), ("h_in", c_int), ("w_in", c_int), ("c_in", c_int),
        ("in_sb", c_ll), ("in_sh", c_ll), ("in_sw", c_ll),
        ("h_out", c_int), ("w_out", c_int), ("n_out", c_int),
        ("kh", c_int), ("kw", c_int), ("sh", c_int), ("sw", c_int),
        ("dh", c_int), ("dw", c_int), ("ph", c_int), ("pw", c_int),
        ("out_sb", c_ll), ("out_sh", c_ll), ("out_sw", c_ll), ("out_sg", c_ll),
        ("n_group", c_int), ("act", c_int), ("prologue", c_int),
        ("pro_stats", c_void_p), ("pro_gamma", c_void_p), ("pro_beta", c_void_p),
        ("pro_group_per_h", c_int), ("pro_x2", c_void_p),
        ("res", c_void_p), ("res_scale", c_void_p),
        ("stats", c_void_p), ("stats_per_h", c_int),
        ("post", c_void_p), ("post_sh", c_ll),
        ("y_bf16", c_int), ("x_bf16", c_int),
    ]


class AttnParams(ctypes.Structure):
    """Mirror of ``UnblendAttnParams``."""

    _fields_ = [
        ("outer", c_int), ("inner", c_int), ("heads", c_int), ("lq", c_int), ("lk", c_int), ("hd", c_int),
        ("q_so", c_ll), ("q_si", c_ll), ("q_sr", c_ll),
        ("kv_so", c_ll), ("kv_si", c_ll), ("kv_sr", c_ll),
        ("out", c_void_p), ("o_so", c_ll), ("o_si", c_ll), ("o_sr", c_ll), ("out_bf16", c_int),
        ("gate", c_void_p), ("g_so", c_ll), ("g_si", c_ll), ("g_sr", c_ll),
        ("rope", c_void_p), ("rope_len", c_int),
        ("scale", c_float),
    ]


class GemmGroup(ctypes.Structure):
    """Mirror of ``UnblendGemmGroup``."""

    _fields_ = [("a_col0", c_int), ("w_row0", c_int), ("n", c_int), ("k", c_int), ("out_col0", c_int)]


class GemmParams(ctypes.Structure):
    """Mirror of ``UnblendGemmParams``."""

    _fields_ = [
        ("groups", c_int), ("group", ctypes.POINTER(GemmGroup)), ("bias", c_void_p), ("act", c_int),
        ("res", c_void_p), ("ldr", c_ll), ("out", c_void_p), ("ldo", c_ll), ("out_bf16", c_int),
        ("rope", c_void_p), ("rope_cols", c_int), ("rope_hd", c_int), ("rope_div", c_int), ("rope_mod", c_int),
    ]


# name -> argtypes (all return int)
_SIGNATURES = {
    "unblend_conv2d_f32": [c_void_p, c_void_p, c_void_p, c_void_p, ctypes.POINTER(ConvParams), c_void_p],
    "unblend_stats_finalize": [c_void_p, c_void_p, c_int, c_double, c_float, c_int, c_int, c_void_p],
    "unblend_zero_f64": [c_void_p, c_ll, c_void_p],
    "unblend_zero_f32": [c_void_p, c_ll, c_int, c_ll, c_void_p],
    "unblend_group_sums": [c_void_p, c_void_p, c_int, c_ll, c_void_p],
    "unblend_group_norm_apply": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_ll, c_int, c_ll, c_int,
                                 c_void_p],
    "unblend_dconv_tail": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_ll, c_ll, c_int,
                           c_ll, c_void_p],
    "unblend_layer_norm": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_ll, c_ll, c_int,
                           c_void_p],
    "unblend_layer_norm_bf16": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_ll, c_ll, c_int,
                                c_void_p],
    "unblend_attention_f32": [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
                              c_ll, c_ll, c_ll, c_ll, c_ll, c_ll, c_float, c_void_p],
    "unblend_add": [c_void_p, c_void_p, c_void_p, c_ll, c_ll, c_float, c_void_p],
    "unblend_standardize": [c_void_p, c_void_p, c_void_p, c_ll, c_int, c_void_p],
    "unblend_stft_cac": [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p],
    "unblend_time_input": [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p],
    "unblend_istft_output": [c_void_p, c_void_p, c_ll, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                             c_int, c_int, c_int, c_int, c_void_p],
    "unblend_mean_std": [c_void_p, c_void_p, c_void_p, c_int, c_ll, c_void_p],
    "unblend_mean_std_noalloc": [c_void_p, c_void_p, c_int, c_ll, c_void_p],
    "unblend_gather_chunks": [c_void_p, c_int, c_ll, c_void_p, c_int, c_int, c_void_p, c_void_p],
    "unblend_overlap_add": [c_void_p, c_int, c_int, c_int, c_void_p, c_ll, c_ll, c_ll, c_float, c_void_p,
                            c_void_p, c_void_p],
    "unblend_weight_chunks": [c_void_p, c_int, c_int, c_int, c_void_p, c_ll, c_float, c_void_p],
    "unblend_divide": [c_void_p, c_void_p, c_void_p, c_int, c_ll, c_void_p],
    "unblend_conv2d_tc": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, ctypes.POINTER(ConvParams), c_int,
                          c_int, c_void_p],
    "unblend_attention_tc": [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_ll, c_ll,
                             c_ll, c_ll, c_ll, c_ll, c_float, c_int, c_void_p],
    "unblend_dconv_conv1": [c_void_p, c_ll, c_int, c_int, c_int, c_void_p, c_void_p, c_int, c_int, c_void_p,
                            c_void_p, c_void_p],
    "unblend_dconv_apply": [c_void_p, c_ll, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p,
                            c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p],
    "unblend_attention_tc2": [c_void_p, c_void_p, c_void_p, ctypes.POINTER(AttnParams), c_int, c_void_p],
    "unblend_attention_bf16": [c_void_p, c_void_p, c_void_p, ctypes.POINTER(AttnParams), c_void_p],
    "unblend_gemm_tc": [c_void_p, c_ll, c_int, c_int, c_void_p, c_void_p, c_ll, c_int, ctypes.POINTER(GemmParams),
                        c_int, c_int, c_void_p],
    "unblend_rms_norm": [c_void_p, c_ll, c_int, c_void_p, c_void_p, c_ll, c_int, c_void_p, c_void_p, c_int,
                         c_void_p, c_void_p],
    "unblend_band_rms_norm": [c_void_p, c_ll, c_ll, c_void_p, c_int, c_void_p, c_void_p, c_ll, c_int, c_void_p,
                              c_void_p],
    "unblend_gather_pairs": [c_void_p, c_ll, c_ll, c_void_p, c_int, c_void_p, c_ll, c_void_p],
    "unblend_cast_bf16": [c_void_p, c_void_p, c_ll, c_void_p],
    "unblend_pcm16_to_f32": [c_void_p, c_int, c_ll, c_void_p, c_int, c_void_p],
    "unblend_convert_channels": [c_void_p, c_int, c_ll, c_void_p, c_int, c_void_p],
    "unblend_resample": [c_void_p, c_int, c_ll, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_ll, c_void_p],
    "unblend_max_abs": [c_void_p, c_ll, c_void_p, c_void_p],
    "unblend_prevent_clip": [c_void_p, c_void_p, c_ll, c_int, c_void_p, c_void_p],
    "unblend_encode_pcm16": [c_void_p, c_int, c_ll, c_int, c_void_p, c_void_p, c_void_p],
    "unblend_dconv_moments": [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                              c_void_p],
    "unblend_dconv_moment_sums": [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p],
    "unblend_scatter_mean_pairs": [c_void_p, c_ll, c_ll, c_void_p, c_void_p, c_int, c_void_p, c_ll, c_void_p],
    "unblend_stft_frames": [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p],
    "unblend_pad_tail": [c_void_p, c_void_p, c_int, c_ll, c_ll, c_void_p],
    "unblend_swap_axes": [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p],
    "unblend_depthwise3": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p],
    "unblend_act_copy": [c_void_p, c_ll, c_void_p, c_ll, c_int, c_ll, c_int, c_void_p],
    "unblend_rfft_time": [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p],
    "unblend_irfft_time": [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p],
    "unblend_lstm_recurrence": [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_ll, c_ll, c_ll, c_void_p],
    "unblend_lstm_recurrence_bf16": [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_ll, c_ll, c_ll,
                                     c_void_p],
    "unblend_lstm_error_flag": [c_void_p, c_int],
    "unblend_istft_masked": [c_void_p, c_void_p, c_ll, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                             c_int, c_int, c_int, c_int, c_void_p],
}

# Entry points without a stream argument.
_HOST_SIGNATURES = {
    "unblend_error_flag": [ctypes.POINTER(c_int), c_int],
    "unblend_attention_error_flag": [ctypes.POINTER(c_int), c_int],
    "unblend_gemm_error_flag": [ctypes.POINTER(c_int), c_int],
    "unblend_attention_bf16_error_flag": [ctypes.POINTER(c_int), c_int],
    "unblend_dconv_error_flag": [ctypes.POINTER(c_int), c_int],
}

# Tensor-core convolution modes (unblend_conv2d_tc): 3-pass TF32, bf16, 3-pass bf16,
# bf16 activations, 3-pass bf16 with the taps of a kernel row sharing one input load.
TC_TF32X3, TC_BF16, TC_BF16X3, TC_BF16_ACT, TC_BF16X3_TAPS = 0, 1, 2, 3, 4

_lib = None


def _check_fresh() -> None:
    """Refuse a library built from other sources than the ones beside it: its
    entry points could take other arguments than the signatures declared here."""
    from .build import CSRC, DIGEST_NAME, source_digest

    if not os.path.isdir(CSRC) or not any(f.endswith(".cu") for f in os.listdir(CSRC)):
        return  # shipped without its sources: nothing to compare against
    stamp = os.path.join(os.path.dirname(LIB_PATH), DIGEST_NAME)
    want = source_digest()
    have = open(stamp).read().strip() if os.path.exists(stamp) else None
    if have != want:
        raise RuntimeError(
            f"unblend_b200 CUDA library {LIB_PATH} was not built from the current sources; "
            "run `python -m unblend_b200.build`"
        )


def load() -> ctypes.CDLL:
    """Load the shared library (once) and declare every entry point."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"unblend_b200 CUDA library not built ({LIB_PATH}); run `python -m unblend_b200.build`"
        )
    _check_fresh()
    lib = ctypes.CDLL(LIB_PATH)
    for name, args in {**_SIGNATURES, **_HOST_SIGNATURES}.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = c_int
    _lib = lib
    return lib


def exported_symbols() -> list[str]:
    """Entry points this binding declares (all must exist in the library)."""
    return list(_SIGNATURES) + list(_HOST_SIGNATURES)


def error_flag(clear: bool = True) -> int:
    """Read (and by default clear) the device flag that bounded waits set on timeout."""
    total = 0
    for name in ("unblend_error_flag", "unblend_attention_error_flag", "unblend_gemm_error_flag",
                 "unblend_attention_bf16_error_flag", "unblend_dconv_error_flag", "unblend_lstm_error_flag"):
        v = c_int(0)
        check(name, getattr(load(), name)(ctypes.byref(v), 1 if clear else 0))
        total |= v.value
    return total


def _cuda_error_string(code: int) -> str:
    try:
        from cuda.bindings import runtime as rt  # type: ignore

        err, name = rt.cudaGetErrorName(rt.cudaError_t(code))
        return name.decode() if isinstance(name, bytes) else str(name)
    except Exception:  # pragma: no cover - best effort text only
        return f"cudaError {code}"


def check(name: str, rc: int) -> None:
    """Raise ``RuntimeError`` for a non-zero launcher return code."""
    if rc == 0:
        return
    if rc == ERR_TOO_LARGE:
        raise RuntimeError(f"{name}: request exceeds the entry point's fixed built-in capacity")
    if rc == ERR_INVALID:
        raise RuntimeError(f"{name}: invalid arguments")
    text = _cuda_error_string(rc)
    if rc == 2:  # cudaErrorMemoryAllocation
        raise RuntimeError(f"CUDA out of memory in {name} ({text})")
    raise RuntimeError(f"{name} failed: {text} ({rc})")


# Kernels launched by one call of each entry point (1 unless listed).
KERNELS_PER_CALL = {"unblend_mean_std": 3, "unblend_istft_output": 2, "unblend_istft_masked": 2}

# Launch accounting: total kernels launched through this binding.
counters = {"launches": 0}

# Optional per-launch timing probe: when a list, each call appends
# (name, start_event, end_event, work) with CUDA events recorded on the
# launching stream around the launch; ``work`` is the caller's algorithmic
# FLOP count for the launch (or None).
probe: list | None = None


def call(name: str, *args, work: float | None = None) -> None:
    """Invoke ``name`` with ``args`` (the trailing stream is appended) and check it."""
    lib = load()
    cur = torch.cuda.current_stream()
    stream = c_void_p(cur.cuda_stream)
    if probe is not None:
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(cur)
        rc = getattr(lib, name)(*args, stream)
        end.record(cur)
        probe.append((name, start, end, work))
    else:
        rc = getattr(lib, name)(*args, stream)
    counters["launches"] += KERNELS_PER_CALL.get(name, 1)
    check(name, rc)


def ptr(t: torch.Tensor | None) -> int | None:
    """Device pointer of a tensor (None stays None)."""
    return None if t is None else t.data_ptr()
