"""ctypes binding of libfry_b200.so, the C ABI declared in include/fry_b200.h.

There is no fallback: if the library is missing or does not load, `library()` raises FryError. Every entry point's
nonzero return becomes a FryError carrying fry_last_error()'s message.
"""
import ctypes
import threading
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIBRARY_PATH = HERE / "libfry_b200.so"

_c_int, _c_float, _ptr, _size = ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t


class FryError(RuntimeError):
    """A refused shape or a failed CUDA call in libfry_b200.so."""


class FryHeads(ctypes.Structure):
    _fields_ = [("ln_gain", _ptr), ("a_weight", _ptr), ("a_bias", _ptr), ("narrow_weight", _ptr), ("narrow_bias", _ptr),
                ("hidden_weight", _ptr), ("hidden_bias", _ptr), ("out_weight", _ptr), ("out_bias", _ptr), ("bins", _c_int)]


class FryBlock(ctypes.Structure):
    _fields_ = [("dq", _c_int), ("ln1", _ptr), ("ln2", _ptr), ("residual_scale", _ptr), ("input_scale", _ptr), ("q_gain", _ptr),
                ("k_gain", _ptr), ("projection", _ptr), ("projection_scale", _ptr), ("projection_bias", _ptr),
                ("combine_heads", _ptr), ("combine_heads_bias", _ptr), ("gate_up", _ptr), ("gate_up_scale", _ptr), ("down", _ptr),
                ("down_scale", _ptr), ("precision", _c_int)]

BLOCK_INT8, BLOCK_FP16 = 0, 1


class FryNetwork(ctypes.Structure):
    _fields_ = [("d_model", _c_int), ("layers", _c_int), ("heads", _c_int), ("kv_heads", _c_int), ("dv", _c_int),
                ("templates_count", _c_int), ("hidden", _c_int), ("down_width", _c_int), ("eps", _c_float), ("embed", _ptr),
                ("position", _ptr), ("table", _ptr), ("templates", _ptr), ("blocks", ctypes.POINTER(FryBlock)),
                ("head_weights", FryHeads)]


class FryLaneHandles(ctypes.Structure):
    _fields_ = [("device", _c_int), ("stream", _ptr), ("done", _ptr), ("rows_host", _ptr), ("rows", _ptr), ("answers_host", _ptr),
                ("answers", _ptr)]


ERROR_SHAPE, ERROR_CUDA, ERROR_STATE = 1, 2, 3

# name -> (argument types, result type); every int-returning entry point is checked
SIGNATURES = {
    "fry_last_error": ([], ctypes.c_char_p),
    "fry_version": ([], ctypes.c_char_p),
    "fry_device_status": ([ctypes.POINTER(_c_int), ctypes.POINTER(_c_int), _c_int], _c_int),
    "fry_set_wait_limit_ns": ([ctypes.c_uint64], _c_int),
    "fry_wait_limit_ns": ([ctypes.POINTER(ctypes.c_uint64)], _c_int),
    "fry_wait_probe": ([_ptr], _c_int),
    "fry_int8_linear": ([_ptr] * 10 + [_c_int] * 4 + [_ptr], _c_int),
    "fry_int8_linear_normed": ([_ptr, _ptr, _c_float] + [_ptr] * 4 + [_c_int] * 4 + [_ptr], _c_int),
    "fry_int8_matmul_i32": ([_ptr] * 3 + [_c_int] * 3 + [_ptr], _c_int),
    "fry_int8_matmul_scaled_bf16": ([_ptr] * 5 + [_c_int] * 3 + [_ptr], _c_int),
    "fry_attention_bf16": ([_ptr] * 4 + [_c_int] * 4 + [_ptr], _c_int),
    "fry_norm_quant": ([_ptr, _ptr, _c_float, _ptr, _ptr, _c_int, _c_int, _ptr], _c_int),
    "fry_mix_norm_quant": ([_ptr] * 5 + [_c_float] + [_ptr] * 3 + [_c_int, _c_int, _ptr], _c_int),
    "fry_rotate_quant": ([_ptr] * 3 + [_c_int] * 3 + [_ptr], _c_int),
    "fry_pair_templates": ([_ptr, _ptr, _c_int, _ptr], _c_int),
    "fry_template_attention": ([_ptr] * 5 + [_c_int] * 6 + [_c_float, _ptr], _c_int),
    "fry_int8_linear_qk_norm": ([_ptr] * 7 + [_c_float, _ptr] + [_c_int] * 6 + [_ptr], _c_int),
    "fry_template_attention_normed": ([_ptr] * 3 + [_c_int] * 6 + [_ptr], _c_int),
    "fry_linear": ([_ptr] * 5 + [_c_int] * 4 + [_ptr], _c_int),
    "fry_linear_full": ([_ptr] * 8 + [_c_int] * 4 + [_ptr], _c_int),
    "fry_linear_norm_quant": ([_ptr] * 6 + [_c_float] + [_ptr] * 2 + [_c_int] * 3 + [_ptr], _c_int),
    "fry_board_embedding": ([_ptr] * 5 + [_c_int, _c_int, _ptr], _c_int),
    "fry_square_feature_rows": ([_ptr, _c_int, _ptr, _ptr], _c_int),
    "fry_heads_workspace_bytes": ([_c_int, _c_int], _size),
    "fry_heads": ([_ptr, ctypes.POINTER(FryHeads), _c_float, _ptr, _ptr, _size, _c_int, _c_int, _ptr], _c_int),
    "fry_heads_noalloc": ([_ptr, ctypes.POINTER(FryHeads), _c_float, _ptr, _c_int, _c_int, _ptr], _c_int),
    "fry_forward_workspace_bytes": ([ctypes.POINTER(FryNetwork), _c_int], _size),
    "fry_forward": ([ctypes.POINTER(FryNetwork), _ptr, _c_int, _ptr, _ptr, _size, _ptr], _c_int),
    "fry_forward_lean_workspace_bytes": ([ctypes.POINTER(FryNetwork), _c_int], _size),
    "fry_forward_lean": ([ctypes.POINTER(FryNetwork), _ptr, _c_int, _ptr, _ptr, _size, _ptr], _c_int),
    "fry_gptq_workspace_bytes": ([_c_int, _c_int], _size),
    "fry_gptq": ([_ptr, _ptr, _c_int, _c_int, _ptr, _ptr, _ptr, _size, _ptr], _c_int),
    "fry_hessian_accumulate": ([_ptr, _c_int, _c_int, _ptr, _ptr], _c_int),
    "fry_lanes_create": ([ctypes.POINTER(FryNetwork), ctypes.POINTER(_c_int), _c_int, _c_int, _c_int, _c_int, ctypes.POINTER(_ptr)], _c_int),
    "fry_lanes_destroy": ([_ptr], _c_int),
    "fry_lanes_free_lane": ([_ptr, ctypes.POINTER(_c_int)], _c_int),
    "fry_lanes_handles": ([_ptr, _c_int, ctypes.POINTER(FryLaneHandles)], _c_int),
    "fry_lanes_graph": ([_ptr, _c_int, _c_int, ctypes.POINTER(_ptr)], _c_int),
    "fry_lanes_launch": ([_ptr, _c_int, _c_int, ctypes.POINTER(_c_int)], _c_int),
    "fry_lanes_collect": ([_ptr, _c_int, ctypes.POINTER(_c_int)], _c_int),
    "fry_lanes_settle": ([_ptr], _c_int),
}

_lock = threading.Lock()
_library = None


class _Library:
    """The loaded library; each attribute is an entry point that raises FryError on a nonzero return."""

    def __init__(self, handle: ctypes.CDLL):
        self.handle = handle
        for name, (arguments, result) in SIGNATURES.items():
            function = getattr(handle, name)
            function.argtypes, function.restype = arguments, result

    def __getattr__(self, name: str):
        function = getattr(self.handle, name)
        if SIGNATURES.get(name, (None, None))[1] is not _c_int or name == "fry_device_status":
            return function

        def checked(*arguments):
            code = function(*arguments)
            if code != 0:
                raise FryError(f"{name}: {self.handle.fry_last_error().decode(errors='replace')}")
            return code
        return checked

    def device_status(self, clear: bool = False) -> tuple[int, int]:
        code, where = _c_int(0), _c_int(0)
        if self.handle.fry_device_status(ctypes.byref(code), ctypes.byref(where), int(clear)) != 0:
            raise FryError(f"fry_device_status: {self.handle.fry_last_error().decode(errors='replace')}")
        return code.value, where.value


def library(path: Path | None = None) -> _Library:
    """The loaded libfry_b200.so (loaded once). Raises FryError if it is missing: build it with build.py."""
    global _library
    with _lock:
        if _library is None:
            target = Path(path) if path is not None else LIBRARY_PATH
            if not target.exists():
                raise FryError(f"{target} is missing: build it with `python chess-transformer_b200/build.py`")
            try:
                _library = _Library(ctypes.CDLL(str(target)))
            except OSError as error:
                raise FryError(f"{target} does not load: {error}") from error
        return _library


def exported_symbols() -> list[str]:
    return list(SIGNATURES)
