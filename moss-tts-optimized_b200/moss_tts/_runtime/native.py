"""ctypes binding of ``libmoss_tts_b200.so``, the C ABI declared in ``include/moss_tts_b200.h``.

The library is built in-tree for sm_100a by ``moss-tts-optimized_b200/build.py``.
There is no fallback: if the library is missing or fails to load, every
operator raises ``NativeLibraryError``. Launch failures (non-zero
``cudaError_t``) raise ``RuntimeError``, as the reference's native launcher
does (``src/moss_tts/_runtime/attention_native.py:41-44``).
"""
import ctypes
import functools
from pathlib import Path

LIB_PATH = Path(__file__).with_name("libmoss_tts_b200.so")
ABI_VERSION = 1
FLAG_PDL = 1
FLAG_REGISTER_PIPELINE = 2
LINEAR_NORM, LINEAR_ADD, LINEAR_PAIRED = 1, 2, 4

_P, _I, _F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
_LLP = ctypes.POINTER(ctypes.c_longlong)

# name -> (argtypes, restype); mirrors include/moss_tts_b200.h
SIGNATURES = {
    "mt_abi_version": ([], _I),
    "mt_read_error_word": ([ctypes.POINTER(ctypes.c_int), _I], _I),
    "mt_dequant_w4": ([_P, _P, _P, _P, _I, _I, _I, _P], _I),
    "mt_static_scales": ([_P, _I, _P, _I, _I, _P], _I),
    "mt_gptq_block": ([_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P], _I),
    "mt_w4a16_linear": ([_P, _P, _P, _F, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P], _I),
    "mt_w4a16_packed_size": ([_I, _I, _I, _I, _LLP, _LLP], _I),
    "mt_w4a16_pack": ([_P, _P, _P, _I, _I, _I, _P, _P], _I),
    "mt_w4a16_linear_packed": ([_P, _P, _P, _F, _P, _P, _I, _P, _I, _I, _I, _P, _I, _P], _I),
    "mt_w4a16_linear_packed_rows": ([_P, _P, _P, _F, _P, _P, _I, _P, _I, _I, _I, _I, _P, _I, _P], _I),
    "mt_w4a16_linear_packed_tp": ([_P, _P, _P, _F, _P, _P, _I, _P, _I, _I, _I, _P, _P, _I, _P], _I),
    "mt_w4a16_gemm_workspace": ([_I, _I, _I, _I, _LLP], _I),
    "mt_w4a16_gemm": ([_P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _I, _P], _I),
    "mt_heads_select": ([_P, _P, _P, _P, _P, _P] + [_I] * 11 + [_P], _I),
    "mt_heads_sample": ([_P] * 8 + [_I] * 10 + [_F, _I, _F, _F, _I, _F, _I, _P], _I),
    "mt_w4a16_gemm_pack_size": ([_I, _I, _I, _LLP], _I),
    "mt_w4a16_gemm_pack": ([_P, _P, _P, _I, _I, _I, _P, _P], _I),
    "mt_w4a16_gemm_packed": ([_P, _P, _P, _I, _I, _I, _I, _P, _I, _P], _I),
    "mt_decode_advance": ([_P, _P, _I, _I, _I, _I, _P], _I),
    "mt_bf16_linear": ([_P, _P, _P, _F, _P, _P, _P, _I, _I, _I, _I, _I, _P], _I),
    "mt_rmsnorm": ([_P, _P, _P, _P, _P, _I, _I, _F, _I, _P], _I),
    "mt_silu_mul": ([_P, _P, _I, _I, _I, _P], _I),
    "mt_embedding_sum": ([_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _I, _P], _I),
    "mt_qk_rope_kv": ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _P, _I, _P], _I),
    "mt_attention_decode": ([_P] * 12 + [_I] * 5 + [_F, _P, _I, _P], _I),
    "mt_attention_decode_noalloc": ([_P] * 9 + [_I] * 5 + [_F, _P, _I, _P], _I),
    "mt_attention_oproj_decode": ([_P] * 10 + [_I, _P, _I, _P, _I, _I, _I, _F, _P, _I, _P], _I),
    "mt_decode_layers_workspace": ([_I, _I, _LLP], _I),
    "mt_decode_layers": ([_P, _I, _I, _I, _P, _P, _P, _P, _I, _F, _P, _P, _P, _P, _I, _P], _I),
    "mt_prefill_qk_rope_kv": ([_P, _P, _P, _P, _P, _I, _P, _P, _P, _I, _I, _I, _I, _F, _I, _P], _I),
    "mt_prefill_attention": ([_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P], _I),
    "mt_heads_greedy": ([_P, _P, _P, _F] + [_P] * 11 + [_I] * 11 + [_P], _I),
}


TP_MAX_RANKS = 8


class TpExchange(ctypes.Structure):
    """``mt_tp_exchange`` of include/moss_tts_b200.h."""
    _fields_ = [("recv", ctypes.c_void_p * TP_MAX_RANKS), ("epoch", ctypes.c_void_p),
                ("world", ctypes.c_int), ("rank", ctypes.c_int), ("in_slot", ctypes.c_int),
                ("out_slot", ctypes.c_int), ("slot_elems", ctypes.c_int)]


class DecodeLayer(ctypes.Structure):
    """``mt_decode_layer`` of include/moss_tts_b200.h."""
    _fields_ = [(name, ctypes.c_void_p) for name in ("qkv", "out", "gate_up", "down", "input_norm", "post_norm",
                                                     "q_norm", "k_norm", "k_cache", "v_cache")]


class NativeLibraryError(RuntimeError):
    """The CUDA library is not built or cannot be loaded; there is no CPU fallback."""


@functools.lru_cache(None)
def library() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise NativeLibraryError(f"{LIB_PATH.name} is not built; run moss-tts-optimized_b200/build.py")
    try:
        lib = ctypes.CDLL(str(LIB_PATH))
    except OSError as exc:
        raise NativeLibraryError(f"cannot load {LIB_PATH}: {exc}") from exc
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    if lib.mt_abi_version() != ABI_VERSION:
        raise NativeLibraryError("libmoss_tts_b200.so ABI version mismatch; rebuild it")
    return lib


def call(name: str, *args) -> None:
    rc = getattr(library(), name)(*args)
    if rc:
        raise RuntimeError(f"{name} failed: CUDA error {rc}")


def error_word(clear: bool = False) -> int:
    """The library's device error word (1 after a kernel gave up a bounded wait)."""
    v = ctypes.c_int(0)
    call("mt_read_error_word", ctypes.byref(v), 1 if clear else 0)
    return v.value


def w4a16_packed_size(n: int, k: int, has_zeros: bool, mode: int) -> tuple[int, int]:
    """(packed weight bytes, workspace bytes) of an [n, k] projection in the packed layout."""
    pb, wb = ctypes.c_longlong(0), ctypes.c_longlong(0)
    call("mt_w4a16_packed_size", n, k, 1 if has_zeros else 0, mode, ctypes.byref(pb), ctypes.byref(wb))
    return pb.value, wb.value


def w4a16_gemm_workspace(batch: int, n: int, k: int, mode: int) -> int:
    """Workspace bytes of mt_w4a16_gemm for this shape on the current device."""
    b = ctypes.c_longlong(0)
    call("mt_w4a16_gemm_workspace", batch, n, k, mode, ctypes.byref(b))
    return b.value


def decode_layers_workspace(n_layers: int, inter: int) -> int:
    """Workspace bytes of mt_decode_layers on the current device."""
    b = ctypes.c_longlong(0)
    call("mt_decode_layers_workspace", n_layers, inter, ctypes.byref(b))
    return b.value


def w4a16_gemm_pack_size(n: int, k: int, mode: int) -> int:
    """Bytes of the batched GEMM's packed layout of an [n, k] projection."""
    b = ctypes.c_longlong(0)
    call("mt_w4a16_gemm_pack_size", n, k, mode, ctypes.byref(b))
    return b.value


def ptr(t) -> int | None:
    """Device address of a tensor (None for a missing optional tensor)."""
    return None if t is None else t.data_ptr()


def stream_of(t) -> int:
    import torch
    return torch.cuda.current_stream(t.device).cuda_stream
