"""ctypes binding of libplm_native.so (declared in include/plm_native.h).

The library is the only compute path: importing this module on a machine without the built library, or calling
into it without an sm_100a GPU, raises ``NativeError``. There is no fallback.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_int32, c_int64, c_size_t, c_void_p, pointer
from pathlib import Path

LIBRARY = Path(__file__).resolve().with_name("libplm_native.so")

PLM_OK = 0
STATUS_NAMES = {-1: "PLM_ERR_INVALID", -2: "PLM_ERR_CUDA", -3: "PLM_ERR_DEVICE", -4: "PLM_ERR_UNSUPPORTED",
                -5: "PLM_ERR_NOMEM"}

PLM_BF16, PLM_F16 = 0, 1
EPI_STORE, EPI_SILU_MUL, EPI_QKV_ROPE, EPI_LOGITS, EPI_TABLE, EPI_PARTIAL = range(6)

DEVICE_ERRORS = {1: "TMA stage wait timed out", 2: "free stage wait timed out", 3: "MMA completion wait timed out",
                 4: "index out of range", 5: "split reduction arrival count inconsistent", 6: "unsupported shape",
                 7: "cluster peer data wait timed out", 8: "cross-CTA operand wait timed out"}


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
                ("table", c_void_p), ("aux", c_int32), ("a0", c_int32),
                ("corr", c_void_p), ("corr_from", c_int32), ("corr_ld", c_int32)]


class GemmDesc(ctypes.Structure):
    _fields_ = [("dtype", c_int32), ("w", c_void_p), ("n_out", c_int32), ("k", c_int32), ("x", c_void_p),
                ("x_rows", c_int32), ("rows", c_int32), ("out", c_void_p), ("ldo", c_int32), ("splits", c_int32),
                ("epi", GemmEpilogue)]


RULE_NUCLEUS, RULE_FLOOR = 0, 1
BOOK_NONE, BOOK_STEADY, BOOK_ROUND0, BOOK_FIRST_TOKEN = range(4)
WEIGHTS_IN_PLACE, WEIGHTS_BLOCK = 1, 2  # plm_borrowed_weights


class Bookkeeping(ctypes.Structure):
    _fields_ = [("mode", c_int32), ("k", c_int32), ("best_val", c_void_p), ("best_idx", c_void_p),
                ("n_tiles", c_int32), ("rows", c_int32), ("out", c_void_p), ("out_cap", c_int64),
                ("base", c_void_p), ("offset", c_void_p), ("anchor", c_void_p), ("pending", c_void_p),
                ("round_sequence", c_void_p), ("seq_cap", c_int64), ("sequence_step", c_void_p),
                ("prompt_len", c_int64), ("stop", c_void_p), ("commit", c_void_p)]


class VerifyDesc(ctypes.Structure):
    _fields_ = [("dtype", c_int32), ("logits", c_void_p), ("n_rows", c_int32), ("vocab", c_int32),
                ("logits_stride", c_int64), ("table", c_void_p), ("aux", c_int32), ("aux_buf", c_void_p),
                ("aux_len", c_int64), ("aux_base", c_void_p), ("aux_row_offset", c_int32), ("pending", c_void_p),
                ("n_accept", c_int32), ("rule", c_int32), ("threshold", ctypes.c_float),
                ("top_m", c_int32), ("shortlist", c_int32), ("rounds", c_int32), ("sweeps", c_int32),
                ("epsilon", ctypes.c_double), ("refocus", ctypes.c_double), ("endpoint", ctypes.c_double),
                ("verify", c_void_p), ("flags", c_void_p), ("dbg_tokens", c_void_p), ("dbg_counts", c_void_p),
                ("dbg_bias", c_void_p), ("dbg_stats", c_void_p), ("dbg_sigma", c_void_p), ("dbg_phase_ns", c_void_p),
                ("book", Bookkeeping)]


class AttentionDesc(ctypes.Structure):
    _fields_ = [("dtype", c_int32), ("q", c_void_p), ("k_cache", c_void_p), ("v_cache", c_void_p),
                ("block_table", c_void_p), ("max_pages", c_int32), ("num_pages", c_int32), ("page_size", c_int32),
                ("offset", c_void_p), ("rows", c_int32), ("depth", c_void_p), ("own_start", c_void_p),
                ("num_heads", c_int32), ("num_kv_heads", c_int32), ("head_dim", c_int32), ("out", c_void_p),
                ("splits", c_int32), ("max_keys", c_int64)]


class KvAppendDesc(ctypes.Structure):
    _fields_ = [("dtype", c_int32), ("k", c_void_p), ("v", c_void_p), ("k_cache", c_void_p), ("v_cache", c_void_p),
                ("block_table", c_void_p), ("max_pages", c_int32), ("num_pages", c_int32), ("page_size", c_int32),
                ("offset", c_void_p), ("rows", c_int32), ("num_kv_heads", c_int32), ("head_dim", c_int32)]


class AddRmsNormDesc(ctypes.Structure):
    _fields_ = [("dtype", c_int32), ("x", c_void_p), ("residual", c_void_p), ("normed", c_void_p),
                ("weight", c_void_p), ("rows", c_int32), ("hidden", c_int32), ("eps", ctypes.c_float),
                ("gather_row", c_int32), ("gathered", c_void_p), ("partials", c_void_p), ("n_partials", c_int32),
                ("partial_stride", ctypes.c_int64), ("corr", c_void_p), ("corr_from", c_int32), ("corr_ld", c_int32)]


class CommitDesc(ctypes.Structure):
    _fields_ = [("dtype", c_int32), ("scratch", c_void_p), ("scratch_rows", c_int32), ("kv_cache", c_void_p),
                ("plane_elems", c_int64), ("layers", c_int32), ("num_kv_heads", c_int32), ("head_dim", c_int32),
                ("page_size", c_int32), ("num_pages", c_int32), ("max_pages", c_int32), ("block_table", c_void_p),
                ("commit", c_void_p)]


class ModelDesc(ctypes.Structure):
    _fields_ = [("dtype", c_int32), ("num_layers", c_int32), ("hidden", c_int32), ("num_heads", c_int32),
                ("num_kv_heads", c_int32), ("head_dim", c_int32), ("intermediate", c_int32), ("vocab", c_int32),
                ("aux_vocab", c_int32), ("num_aux_tokens", c_int32), ("rms_eps", ctypes.c_float),
                ("max_pos", c_int32), ("top_m", c_int32), ("shortlist", c_int32), ("rounds", c_int32),
                ("sweeps", c_int32), ("epsilon", ctypes.c_double), ("refocus", ctypes.c_double),
                ("endpoint", ctypes.c_double)]


class IcdfDesc(ctypes.Structure):
    _fields_ = [("logits", c_void_p), ("ld", c_int64), ("u", c_void_p), ("n_rows", c_int32), ("vocab", c_int32),
                ("top_k", c_int32), ("tokens", c_void_p), ("ids_out", c_void_p), ("edges_out", c_void_p)]


class PtpDesc(ctypes.Structure):
    _fields_ = [("embedding", c_void_p), ("num_embeddings", c_int32), ("top_k", c_int32), ("rank", c_int32),
                ("qkv_a", POINTER(c_void_p)), ("qkv_b", POINTER(c_void_p)), ("o_a", POINTER(c_void_p)),
                ("o_b", POINTER(c_void_p)), ("gate_up_a", POINTER(c_void_p)), ("gate_up_b", POINTER(c_void_p)),
                ("down_a", POINTER(c_void_p)), ("down_b", POINTER(c_void_p))]


class WeightPtrs(ctypes.Structure):
    _fields_ = [("embed", c_void_p), ("lm_head", c_void_p), ("final_norm", c_void_p), ("aux_vocab", c_void_p),
                ("mask_aux", c_void_p), ("cos_sin", c_void_p), ("qkv", POINTER(c_void_p)), ("o", POINTER(c_void_p)),
                ("gate_up", POINTER(c_void_p)), ("down", POINTER(c_void_p)), ("input_norm", POINTER(c_void_p)),
                ("post_norm", POINTER(c_void_p)), ("table", c_void_p), ("ptp", POINTER(PtpDesc))]


class RoundDesc(ctypes.Structure):
    _fields_ = [("k", c_int32), ("rule", c_int32), ("threshold", ctypes.c_float), ("page_size", c_int32),
                ("num_pages", c_int32), ("max_pages", c_int32), ("out_capacity", c_int64),
                ("seq_capacity", c_int64), ("aux_len", c_int64), ("max_prefill", c_int32),
                ("separate_mlp", c_int32)]


class StatePtrs(ctypes.Structure):
    _fields_ = [("out", c_void_p), ("base", c_void_p), ("offset", c_void_p), ("anchor", c_void_p),
                ("pending", c_void_p), ("round_sequence", c_void_p), ("sequence_step", c_void_p),
                ("aux_buf", c_void_p), ("block_table", c_void_p), ("verify_logits", c_void_p),
                ("best_val", c_void_p), ("best_idx", c_void_p), ("verify", c_void_p), ("flags", c_void_p),
                ("hidden_normed", c_void_p), ("kv_cache", c_void_p), ("table", c_void_p),
                ("out_capacity", c_int64), ("seq_capacity", c_int64), ("aux_len", c_int64), ("plane_elems", c_int64),
                ("width", c_int32), ("lm_tiles", c_int32), ("row_capacity", c_int32), ("stop", c_void_p),
                ("round_kv", c_void_p), ("commit", c_void_p)]


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
    "plm_verify_decode_static": [POINTER(VerifyDesc), c_void_p, c_void_p],
    "plm_attention": [c_void_p, POINTER(AttentionDesc), c_void_p],
    "plm_kv_append": [c_void_p, POINTER(KvAppendDesc), c_void_p],
    "plm_add_rmsnorm": [c_void_p, POINTER(AddRmsNormDesc), c_void_p],
    "plm_commit": [c_void_p, POINTER(CommitDesc), c_void_p],
    "plm_icdf_decode": [c_void_p, POINTER(IcdfDesc), c_void_p],
    "plm_block_schedule": [c_int32, c_int32, c_int32, c_int32, POINTER(c_int32), c_int32, POINTER(c_int32),
                           POINTER(c_int32)],
    "plm_create": [POINTER(ModelDesc), POINTER(WeightPtrs), POINTER(RoundDesc), POINTER(c_void_p)],
    "plm_destroy": [c_void_p],
    "plm_set_block_table": [c_void_p, POINTER(c_int32), c_int32],
    "plm_set_aux_stream": [c_void_p, c_void_p, c_int64, c_void_p],
    "plm_set_aux_uniforms": [c_void_p, c_void_p, c_int64, c_void_p],
    "plm_load_prompt": [c_void_p, c_void_p, c_int64, c_void_p],
    "plm_set_stop": [c_void_p, c_int64, c_int64, c_int64, c_void_p],
    "plm_prefill": [c_void_p, c_void_p],
    "plm_round0": [c_void_p, c_void_p],
    "plm_round": [c_void_p, c_void_p],
    "plm_layer_block": [c_void_p, c_int32, c_int32, c_void_p],
    "plm_borrowed_weights": [c_void_p, ctypes.POINTER(c_int32)],
    "plm_state": [c_void_p, POINTER(StatePtrs)],
    "plm_check": [c_void_p, POINTER(c_int32)],
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
    """Enqueue plm_verify_decode (one cluster of 8 CTAs per verify row)."""
    check(library().plm_verify_decode(ctx.handle, ctypes.byref(desc), stream_handle(stream)), "plm_verify_decode")


def attention(ctx: Context, desc: AttentionDesc, stream=None) -> None:
    check(library().plm_attention(ctx.handle, ctypes.byref(desc), stream_handle(stream)), "plm_attention")


def kv_append(ctx: Context, desc: KvAppendDesc, stream=None) -> None:
    check(library().plm_kv_append(ctx.handle, ctypes.byref(desc), stream_handle(stream)), "plm_kv_append")


def add_rmsnorm(ctx: Context, desc: AddRmsNormDesc, stream=None) -> None:
    check(library().plm_add_rmsnorm(ctx.handle, ctypes.byref(desc), stream_handle(stream)), "plm_add_rmsnorm")


def commit(ctx: Context, desc: CommitDesc, stream=None) -> None:
    """Enqueue plm_commit: the rows the device commit record names, from round scratch into the paged cache."""
    check(library().plm_commit(ctx.handle, ctypes.byref(desc), stream_handle(stream)), "plm_commit")


def block_schedule(num_sms: int, hidden: int, intermediate: int, q_size: int) -> list[list[int]]:
    """The layer block's unit codes per CTA (host only; see plm_block_schedule)."""
    lib = library()
    n = c_int32(0)
    offsets = (c_int32 * (num_sms + 1))()
    status = lib.plm_block_schedule(num_sms, hidden, intermediate, q_size, None, 0, offsets, ctypes.byref(n))
    if status != 0 and n.value == 0:
        check(status, "plm_block_schedule")
    units = (c_int32 * n.value)()
    check(lib.plm_block_schedule(num_sms, hidden, intermediate, q_size, units, n.value, offsets, ctypes.byref(n)),
          "plm_block_schedule")
    return [list(units[offsets[c]:offsets[c + 1]]) for c in range(num_sms)]


def icdf_decode(ctx: Context, logits, u, top_k: int, tokens, ids_out=None, edges_out=None, stream=None) -> None:
    """The PTP scheme's inverse-CDF verify decode of ``logits`` ([rows, vocab] float32 on the device) at the
    uniforms ``u`` ([rows] float32) into ``tokens`` ([rows] int64); optionally the chosen ids and bin edges."""
    desc = IcdfDesc(logits=logits.data_ptr(), ld=logits.stride(0), u=u.data_ptr(), n_rows=logits.shape[0],
                    vocab=logits.shape[1], top_k=top_k, tokens=tokens.data_ptr(),
                    ids_out=None if ids_out is None else ids_out.data_ptr(),
                    edges_out=None if edges_out is None else edges_out.data_ptr())
    check(library().plm_icdf_decode(ctx.handle, ctypes.byref(desc), stream_handle(stream)), "plm_icdf_decode")


class _DeviceArray:
    """A zero-copy torch view of device memory owned by a handle (``__cuda_array_interface__``)."""

    def __init__(self, address: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (address, False), "version": 3,
                                         "strides": None}


def device_view(address: int, shape: tuple, dtype):
    """torch tensor aliasing ``shape`` elements of ``dtype`` at a device address (no copy, not owned)."""
    import torch

    typestr = {torch.int64: "<i8", torch.int32: "<i4", torch.float32: "<f4", torch.float16: "<f2",
               torch.bfloat16: "<V2"}[dtype]
    if dtype == torch.bfloat16:
        raw = torch.as_tensor(_DeviceArray(address, shape, "<i2"), device="cuda")
        return raw.view(torch.bfloat16)
    return torch.as_tensor(_DeviceArray(address, shape, typestr), device="cuda")


class Handle:
    """A plm_handle: the round engine of one request stream on the current GPU."""

    def __init__(self, model: ModelDesc, weights: WeightPtrs, round_desc: RoundDesc, keepalive=()) -> None:
        handle = c_void_p()
        self._keepalive = keepalive  # weight pointer arrays and tensors the handle borrows
        check(library().plm_create(ctypes.byref(model), ctypes.byref(weights), ctypes.byref(round_desc),
                                   ctypes.byref(handle)), "plm_create")
        self.handle = handle
        self.model, self.round_desc = model, round_desc

    def state(self) -> StatePtrs:
        p = StatePtrs()
        check(library().plm_state(self.handle, ctypes.byref(p)), "plm_state")
        return p

    def set_block_table(self, table) -> None:
        arr = (c_int32 * len(table))(*[int(v) for v in table])
        check(library().plm_set_block_table(self.handle, arr, len(table)), "plm_set_block_table")

    def set_aux_stream(self, cells, stream=None) -> None:
        check(library().plm_set_aux_stream(self.handle, cells.data_ptr(), cells.numel(), stream_handle(stream)),
              "plm_set_aux_stream")

    def set_aux_uniforms(self, u, stream=None) -> None:
        """The PTP scheme's uniform stream (float32 device or pinned tensor)."""
        check(library().plm_set_aux_uniforms(self.handle, u.data_ptr(), u.numel(), stream_handle(stream)),
              "plm_set_aux_uniforms")

    def load_prompt(self, ids, stream=None) -> None:
        check(library().plm_load_prompt(self.handle, ids.data_ptr(), ids.numel(), stream_handle(stream)),
              "plm_load_prompt")

    def set_stop(self, max_tokens: int, eos_token: int | None = None, eos_window: int = 0, stream=None) -> None:
        """The request's stop block (plm_set_stop): budget, end-of-text id (None: none) and its window."""
        check(library().plm_set_stop(self.handle, int(max_tokens), -1 if eos_token is None else int(eos_token),
                                     int(eos_window), stream_handle(stream)), "plm_set_stop")

    def prefill(self, stream=None) -> None:
        check(library().plm_prefill(self.handle, stream_handle(stream)), "plm_prefill")

    def round0(self, stream=None) -> None:
        check(library().plm_round0(self.handle, stream_handle(stream)), "plm_round0")

    def round(self, stream=None) -> None:
        check(library().plm_round(self.handle, stream_handle(stream)), "plm_round")

    def borrowed_weights(self) -> int:
        """Bit mask of the caller's weight groups the handle still reads (WEIGHTS_IN_PLACE, WEIGHTS_BLOCK)."""
        groups = c_int32(0)
        check(library().plm_borrowed_weights(self.handle, ctypes.byref(groups)), "plm_borrowed_weights")
        return groups.value

    def layer_block(self, layer: int, rows: int, stream=None) -> None:
        """One decoder layer's o projection, post-attention norm and MLP as the round runs it (plm_layer_block)."""
        check(library().plm_layer_block(self.handle, layer, rows, stream_handle(stream)), "plm_layer_block")

    def check(self) -> None:
        code = c_int32(0)
        check(library().plm_check(self.handle, ctypes.byref(code)), "plm_check")
        if code.value:
            raise NativeError(f"device error {code.value}: {DEVICE_ERRORS.get(code.value, 'unknown')}")

    def close(self) -> None:
        if getattr(self, "handle", None):
            library().plm_destroy(self.handle)
            self.handle = c_void_p()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass
