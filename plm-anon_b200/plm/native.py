"""ctypes binding of libplm_native.so (declared in include/plm_native.h).

The library is the only compute path: importing this module on a machine without the built library, or calling
into it without an sm_100a GPU, raises ``NativeError``. There is no fallback.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_int32, c_int64, c_size_t, c_void_p
from pathlib import Path

LIBRARY = Path(__file__).resolve().with_name("libplm_native.so")

PLM_OK = 0
STATUS_NAMES = {-1: "PLM_ERR_INVALID", -2: "PLM_ERR_CUDA", -3: "PLM_ERR_DEVICE", -4: "PLM_ERR_UNSUPPORTED",
                -5: "PLM_ERR_NOMEM"}

PLM_BF16, PLM_F16 = 0, 1
EPI_STORE, EPI_SILU_MUL, EPI_QKV_ROPE, EPI_LOGITS, EPI_TABLE = range(5)

DEVICE_ERRORS = {1: "TMA stage wait timed out", 2: "free stage wait timed out", 3: "MMA completion wait timed out",
                 4: "index out of range", 5: "split reduction arrival count inconsistent", 6: "unsupported shape"}


class NativeError(RuntimeError):
    pass


class GemmEpilogue(ctypes.Structure):
    _fields_ = [("kind", c_int32), ("gate_offset", c_int32),
                ("q_out", c_void_p), ("k_cache", c_void_p), ("v_cache", c_void_p), ("positions", c_void_p),
                ("slots", c_void_p), ("cos_sin", c_void_p),
                ("num_heads", c_int32), ("num_kv_heads", c_int32), ("head_dim", c_int32), ("page_size", c_int32),
                ("num_slots", c_int64), ("max_pos", c_int32),
                ("verify_logits", c_void_p), ("best_val", c_void_p), ("best_idx", c_void_p),
                ("n_verify", c_int32), ("vocab", c_int32),
                ("table", c_void_p), ("aux", c_int32), ("a0", c_int32)]


class GemmDesc(ctypes.Structure):
    _fields_ = [("dtype", c_int32), ("w", c_void_p), ("n_out", c_int32), ("k", c_int32), ("x", c_void_p),
                ("x_rows", c_int32), ("rows", c_int32), ("out", c_void_p), ("ldo", c_int32), ("splits", c_int32),
                ("epi", GemmEpilogue)]


RULE_NUCLEUS, RULE_FLOOR = 0, 1
BOOK_NONE, BOOK_STEADY, BOOK_ROUND0, BOOK_FIRST_TOKEN = range(4)


class Bookkeeping(ctypes.Structure):
    _fields_ = [("mode", c_int32), ("k", c_int32), ("best_val", c_void_p), ("best_idx", c_void_p),
                ("n_tiles", c_int32), ("rows", c_int32), ("out", c_void_p), ("out_cap", c_int64),
                ("base", c_void_p), ("offset", c_void_p), ("anchor", c_void_p), ("pending", c_void_p),
                ("round_sequence", c_void_p), ("seq_cap", c_int64), ("sequence_step", c_void_p),
                ("prompt_len", c_int64)]


class VerifyDesc(ctypes.Structure):
    _fields_ = [("dtype", c_int32), ("logits", c_void_p), ("n_rows", c_int32), ("vocab", c_int32),
                ("logits_stride", c_int64), ("table", c_void_p), ("aux", c_int32), ("aux_buf", c_void_p),
                ("aux_len", c_int64), ("aux_base", c_void_p), ("aux_row_offset", c_int32), ("pending", c_void_p),
                ("n_accept", c_int32), ("rule", c_int32), ("threshold", ctypes.c_float),
                ("top_m", c_int32), ("shortlist", c_int32), ("rounds", c_int32), ("sweeps", c_int32),
                ("epsilon", ctypes.c_double), ("refocus", ctypes.c_double), ("endpoint", ctypes.c_double),
                ("verify", c_void_p), ("flags", c_void_p), ("dbg_tokens", c_void_p), ("dbg_counts", c_void_p),
                ("dbg_bias", c_void_p), ("dbg_stats", c_void_p), ("dbg_sigma", c_void_p), ("book", Bookkeeping)]


_lib: ctypes.CDLL | None = None

# name -> (argtypes); every entry point returns int
_SIGNATURES: dict[str, list] = {
    "plm_abi_version": [],
    "plm_last_error": [c_char_p, c_size_t],
    "plm_ctx_create": [POINTER(c_void_p)],
    "plm_ctx_destroy": [c_void_p],
    "plm_ctx_check": [c_void_p, POINTER(c_int32)],
    "plm_gemm_tiles": [c_int32, c_int32, c_int32, POINTER(c_int32)],
    "plm_gemm": [c_void_p, POINTER(GemmDesc), c_void_p],
    "plm_verify_decode": [c_void_p, POINTER(VerifyDesc), c_void_p],
}


def library() -> ctypes.CDLL:
    """The loaded library with every entry point's signature declared."""
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            raise NativeError(f"{LIBRARY} is missing: build it with plm-anon_b200/csrc/build.py")
        lib = ctypes.CDLL(str(LIBRARY))
        for name, argtypes in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = c_int32
        _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    library().plm_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int, what: str) -> None:
    if status != PLM_OK:
        raise NativeError(f"{what}: {STATUS_NAMES.get(status, status)}: {last_error()}")


def ptr(tensor) -> int | None:
    """Device address of a torch tensor (None for None)."""
    return None if tensor is None else tensor.data_ptr()


def stream_handle(stream=None) -> int:
    import torch

    stream = stream if stream is not None else torch.cuda.current_stream()
    return stream.cuda_stream


class Context:
    """A plm_ctx: the device error word and split-reduction scratch of the current device."""

    def __init__(self) -> None:
        handle = c_void_p()
        check(library().plm_ctx_create(ctypes.byref(handle)), "plm_ctx_create")
        self.handle = handle

    def check(self) -> None:
        """Synchronise and raise if any kernel recorded a device error since the last check."""
        code = c_int32(0)
        check(library().plm_ctx_check(self.handle, ctypes.byref(code)), "plm_ctx_check")
        if code.value:
            raise NativeError(f"device error {code.value}: {DEVICE_ERRORS.get(code.value, 'unknown')}")

    def close(self) -> None:
        if self.handle:
            library().plm_ctx_destroy(self.handle)
            self.handle = c_void_p()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass


def gemm_tiles(kind: int, n_out: int, gate_offset: int = 0) -> int:
    tiles = c_int32(0)
    check(library().plm_gemm_tiles(kind, n_out, gate_offset, ctypes.byref(tiles)), "plm_gemm_tiles")
    return tiles.value


def gemm(ctx: Context, w, x, rows: int, *, out=None, epi: GemmEpilogue | None = None, splits: int = 0,
         stream=None) -> None:
    """Enqueue Y = X[:rows] . W^T with the given epilogue (default: store into ``out``)."""
    import torch

    if w.dtype != torch.bfloat16 or x.dtype != torch.bfloat16:
        raise NativeError("plm_gemm: bf16 operands required")
    epi = epi if epi is not None else GemmEpilogue(kind=EPI_STORE)
    desc = GemmDesc(dtype=PLM_BF16, w=ptr(w), n_out=w.shape[0], k=w.shape[1], x=ptr(x), x_rows=x.shape[0],
                    rows=rows, out=ptr(out), ldo=(out.stride(0) if out is not None else 0), splits=splits, epi=epi)
    check(library().plm_gemm(ctx.handle, ctypes.byref(desc), stream_handle(stream)), "plm_gemm")


def verify_decode(ctx: Context, desc: VerifyDesc, stream=None) -> None:
    """Enqueue plm_verify_decode (one CTA per row)."""
    check(library().plm_verify_decode(ctx.handle, ctypes.byref(desc), stream_handle(stream)), "plm_verify_decode")
