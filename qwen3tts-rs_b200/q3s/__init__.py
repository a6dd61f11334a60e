"""Python binding of the B200 sampler C ABI (include/q3s_sampler.h).

The product path is the CUDA library lib/libq3s_sampler.so; this module only
marshals arguments through ctypes.  Loading fails loudly when the library is
missing: there is no CPU fallback.

Surface mirrored from the reference (qwen3tts-rs src/talker/sampling.rs):
    SamplingOptions            sampling.rs:19-25, greedy() :133-142
    Sampler                    sampling.rs:144-335 (sample, sample_with_mode,
                               sample_with_transfer_observer,
                               sample_with_mode_and_transfer_observer,
                               subsequence_counter, diagnostics)
    greedy_select_on_device    sampling.rs:72-117
    greedy_select              sampling.rs:40-60 (on device, many rows)
plus the batched entry point `sample_batch`, one fused launch over many rows.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from pathlib import Path
from typing import Callable, Optional, Sequence

import numpy as np

PKG = Path(__file__).resolve().parent.parent
LIB_PATH = PKG / "lib" / "libq3s_sampler.so"

OK = 0
E_INVALID_ARGUMENT = -1
E_CUDA = -2
E_NO_DEVICE = -3
E_OUT_OF_MEMORY = -4
E_SAMPLING = -5

STATUS_OK = 0
STATUS_INVALID_REPETITION_PENALTY = 1
STATUS_INVALID_TEMPERATURE = 2
STATUS_INVALID_TOP_P = 3
STATUS_SUPPRESSION_NO_CANDIDATE = 4
STATUS_NO_CANDIDATE = 5
STATUS_INVALID_DENOMINATOR = 6
STATUS_UNSUPPORTED = 7
STATUS_INVALID_CODE = 8
STATUS_HISTORY_FULL = 9
MAX_CODE_GROUPS = 32
MAX_VOCAB = 4096

DTYPE_F32 = 0
DTYPE_BF16 = 1
NONE = -1
GREEDY_SELECT = 0
GREEDY_ON_DEVICE = 1
TRANSFER_SAMPLED_TOKEN = 0

# q3s_row_params (48 bytes).
ROW_PARAMS_DTYPE = np.dtype([
    ("temperature", "<f8"), ("top_p", "<f8"), ("repetition_penalty", "<f8"),
    ("top_k", "<u4"), ("do_sample", "<u4"), ("suppress_from", "<i4"),
    ("allow_token", "<i4"), ("ctr_lo", "<u4"), ("reserved", "<u4"),
])
assert ROW_PARAMS_DTYPE.itemsize == 48


class SamplingError(RuntimeError):
    """A sampling call failed; `status` is the Q3S_STATUS_* of the row."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class LibraryError(RuntimeError):
    pass


class _Options(ctypes.Structure):
    _fields_ = [("temperature", ctypes.c_double), ("top_k", ctypes.c_uint64),
                ("top_p", ctypes.c_double), ("repetition_penalty", ctypes.c_double)]


class _Batch(ctypes.Structure):
    _fields_ = [
        ("logits", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("vocab", ctypes.c_int32),
        ("num_rows", ctypes.c_int64), ("row_stride", ctypes.c_int64),
        ("row_offsets", ctypes.c_void_p), ("row_vocab", ctypes.c_void_p),
        ("params", ctypes.c_void_p), ("params_stride", ctypes.c_int64),
        ("seeds", ctypes.c_void_p), ("subseqs", ctypes.c_void_p),
        ("history", ctypes.c_void_p), ("history_offsets", ctypes.c_void_p),
        ("tokens", ctypes.c_void_p), ("status", ctypes.c_void_p),
        ("uniform_override", ctypes.c_void_p), ("probs", ctypes.c_void_p),
        ("masks", ctypes.c_void_p), ("probs_stride", ctypes.c_int64),
        ("history_ends", ctypes.c_void_p),
    ]


class _HeadBatch(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_void_p), ("hidden_dtype", ctypes.c_int32),
        ("hidden_size", ctypes.c_int32), ("hidden_stride", ctypes.c_int64),
        ("weight", ctypes.c_void_p), ("logits", ctypes.c_void_p), ("sample", _Batch),
    ]


class _SessionConfig(ctypes.Structure):
    _fields_ = [
        ("id", ctypes.c_uint64), ("seed", ctypes.c_uint64), ("subseq", ctypes.c_uint64),
        ("talker", _Options), ("predictor", _Options),
        ("talker_do_sample", ctypes.c_int32), ("predictor_do_sample", ctypes.c_int32),
        ("suppress_from", ctypes.c_int32), ("allow_token", ctypes.c_int32),
        ("history", ctypes.c_void_p), ("history_len", ctypes.c_int64),
    ]


class _Commit(ctypes.Structure):
    _fields_ = [
        ("num_rows", ctypes.c_int64), ("params", ctypes.c_void_p),
        ("params_stride", ctypes.c_int64), ("tokens", ctypes.c_void_p),
        ("status", ctypes.c_void_p), ("subseqs", ctypes.c_void_p), ("codes", ctypes.c_void_p),
        ("codes_stride", ctypes.c_int64), ("group", ctypes.c_int32),
        ("reserved", ctypes.c_int32), ("frame_status", ctypes.c_void_p),
        ("history", ctypes.c_void_p), ("history_ends", ctypes.c_void_p),
        ("history_limits", ctypes.c_void_p),
    ]


class _EmbedBatch(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int32), ("groups", ctypes.c_int32), ("hidden", ctypes.c_int32),
        ("reserved", ctypes.c_int32), ("num_rows", ctypes.c_int64), ("codes", ctypes.c_void_p),
        ("tables", ctypes.c_void_p), ("vocab", ctypes.c_void_p), ("text", ctypes.c_void_p),
        ("text_stride", ctypes.c_int64), ("out", ctypes.c_void_p), ("status", ctypes.c_void_p),
    ]


class _Diagnostics(ctypes.Structure):
    _fields_ = [("call_count", ctypes.c_uint32), ("sampled_calls", ctypes.c_uint32),
                ("greedy_calls", ctypes.c_uint32), ("history_nonempty_calls", ctypes.c_uint32),
                ("history_nonempty_sequence", ctypes.c_uint8 * 64),
                ("sequence", ctypes.c_uint8 * 64), ("sequence_len", ctypes.c_uint64)]


TRANSFER_CALLBACK = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
                                     ctypes.c_uint64)

# Every symbol include/q3s_sampler.h declares.
EXPORTED_SYMBOLS = (
    "q3s_abi_version", "q3s_last_error", "q3s_status_message", "q3s_context_create",
    "q3s_context_destroy", "q3s_sample_batch", "q3s_greedy_batch", "q3s_sampler_create",
    "q3s_sampler_destroy", "q3s_sampler_subsequence_counter",
    "q3s_sampler_set_subsequence_counter", "q3s_sampler_get_diagnostics",
    "q3s_sampler_sample_with_mode", "q3s_sampler_sample", "q3s_sample_batch_static",
    "q3s_embed_sum", "q3s_context_set_test_hooks", "q3s_context_set_path_stats",
    "q3s_commit_rows", "q3s_scheduler_create", "q3s_scheduler_destroy", "q3s_scheduler_add",
    "q3s_scheduler_cancel", "q3s_scheduler_begin_frame", "q3s_scheduler_step",
    "q3s_scheduler_end_frame", "q3s_scheduler_codes", "q3s_scheduler_session_state",
    "q3s_head_sample", "q3s_sample_commit",
)

HEAD_MAX_ROWS = 16

# Row paths of the sampling kernel (Q3S_PATH_* of include/q3s_sampler.h).
PATH_NAMES = (
    "invalid", "greedy", "topk", "topk_topp", "front_done", "nucleus", "general_rules",
    "general_inf", "general_tau", "general_overflow", "general_wide", "general_nucleus",
)

_lib = None


def load(path: Optional[os.PathLike] = None):
    """Loads the CUDA sampler library (building it first when nvcc is here)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        import importlib.util
        spec = importlib.util.spec_from_file_location("_q3s_build", PKG / "build.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        try:
            mod.build()
        except Exception as exc:  # no toolkit: fail loudly, never fall back
            raise LibraryError(f"sampler library missing at {p} and it cannot be built: {exc}")
    L = ctypes.CDLL(str(p))
    L.q3s_abi_version.restype = ctypes.c_int
    L.q3s_last_error.restype = ctypes.c_char_p
    L.q3s_status_message.restype = ctypes.c_char_p
    L.q3s_status_message.argtypes = [ctypes.c_int]
    L.q3s_context_create.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]
    L.q3s_context_destroy.argtypes = [ctypes.c_void_p]
    L.q3s_context_destroy.restype = None
    L.q3s_context_set_test_hooks.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int32]
    L.q3s_context_set_path_stats.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    L.q3s_sample_batch.argtypes = [ctypes.c_void_p, ctypes.POINTER(_Batch), ctypes.c_void_p]
    L.q3s_sample_batch_static.argtypes = [ctypes.c_void_p, ctypes.POINTER(_Batch),
                                          ctypes.c_void_p]
    L.q3s_embed_sum.argtypes = [ctypes.c_void_p, ctypes.POINTER(_EmbedBatch), ctypes.c_void_p]
    L.q3s_commit_rows.argtypes = [ctypes.c_void_p, ctypes.POINTER(_Commit), ctypes.c_void_p]
    L.q3s_head_sample.argtypes = [ctypes.c_void_p, ctypes.POINTER(_HeadBatch), ctypes.c_void_p]
    L.q3s_sample_commit.argtypes = [ctypes.c_void_p, ctypes.POINTER(_Batch),
                                    ctypes.POINTER(_Commit), ctypes.c_void_p]
    L.q3s_scheduler_create.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
                                       ctypes.c_int64, ctypes.POINTER(ctypes.c_void_p)]
    L.q3s_scheduler_destroy.argtypes = [ctypes.c_void_p]
    L.q3s_scheduler_destroy.restype = None
    L.q3s_scheduler_add.argtypes = [ctypes.c_void_p, ctypes.POINTER(_SessionConfig)]
    L.q3s_scheduler_cancel.argtypes = [ctypes.c_void_p, ctypes.c_uint64]
    L.q3s_scheduler_begin_frame.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint64),
                                            ctypes.c_int32, ctypes.POINTER(ctypes.c_int32),
                                            ctypes.c_void_p]
    L.q3s_scheduler_step.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p,
                                     ctypes.c_int32, ctypes.c_int32, ctypes.c_int64,
                                     ctypes.c_void_p]
    L.q3s_scheduler_end_frame.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                          ctypes.c_void_p]
    L.q3s_scheduler_codes.argtypes = [ctypes.c_void_p]
    L.q3s_scheduler_codes.restype = ctypes.c_void_p
    L.q3s_scheduler_session_state.argtypes = [ctypes.c_void_p, ctypes.c_uint64,
                                              ctypes.POINTER(ctypes.c_uint64),
                                              ctypes.POINTER(ctypes.c_int64), ctypes.c_void_p,
                                              ctypes.c_int64]
    L.q3s_greedy_batch.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
                                   ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
                                   ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
                                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    L.q3s_sampler_create.argtypes = [ctypes.c_void_p, ctypes.c_uint64,
                                     ctypes.POINTER(ctypes.c_void_p)]
    L.q3s_sampler_destroy.argtypes = [ctypes.c_void_p]
    L.q3s_sampler_destroy.restype = None
    L.q3s_sampler_subsequence_counter.argtypes = [ctypes.c_void_p]
    L.q3s_sampler_subsequence_counter.restype = ctypes.c_uint64
    L.q3s_sampler_set_subsequence_counter.argtypes = [ctypes.c_void_p, ctypes.c_uint64]
    L.q3s_sampler_set_subsequence_counter.restype = None
    L.q3s_sampler_get_diagnostics.argtypes = [ctypes.c_void_p, ctypes.POINTER(_Diagnostics)]
    L.q3s_sampler_sample_with_mode.argtypes = [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
        ctypes.POINTER(_Options), ctypes.c_int32, ctypes.c_int64, ctypes.c_int64,
        ctypes.c_void_p, ctypes.c_int64, TRANSFER_CALLBACK, ctypes.c_void_p,
        ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_int32), ctypes.c_void_p]
    L.q3s_sampler_sample.argtypes = [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
        ctypes.POINTER(_Options), ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
        ctypes.c_int64, ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_int32),
        ctypes.c_void_p]
    if path is None:
        _lib = L
    return L


def last_error() -> str:
    return load().q3s_last_error().decode()


def status_message(status: int) -> str:
    return load().q3s_status_message(int(status)).decode()


def _check(rc: int, what: str) -> None:
    if rc != OK:
        raise LibraryError(f"{what} failed ({rc}): {last_error()}")


@dataclass(frozen=True)
class SamplingOptions:
    """SamplingOptions (sampling.rs:19-25)."""
    temperature: float
    top_k: int
    top_p: float
    repetition_penalty: float

    @staticmethod
    def greedy() -> "SamplingOptions":
        return SamplingOptions(0.0, 0, 1.0, 1.0)

    def _c(self) -> _Options:
        return _Options(float(self.temperature), int(self.top_k), float(self.top_p),
                        float(self.repetition_penalty))


def _none(v) -> int:
    return NONE if v is None else int(v)


class Context:
    """A q3s_context on one device (one per device and host thread)."""

    def __init__(self, device: int = 0):
        self.device = int(device)
        self._h = ctypes.c_void_p()
        _check(load().q3s_context_create(self.device, ctypes.byref(self._h)),
               "q3s_context_create")

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    def set_test_hooks(self, stage_wait_ns: int = 0, hold_refill: bool = False) -> None:
        """Testing hook (q3s_context_set_test_hooks): the per-row stage-wait
        limit of this context's batched launches (0 = the default second) and
        whether ring stages are refilled after their first row."""
        _check(load().q3s_context_set_test_hooks(self._h, int(stage_wait_ns),
                                                 1 if hold_refill else 0),
               "q3s_context_set_test_hooks")

    def set_path_stats(self, stats) -> None:
        """Diagnostics (q3s_context_set_path_stats): `stats` is an int64
        device tensor of 2 * len(PATH_NAMES) entries that this context's
        batched launches accumulate into (rows, then warp cycles, per path),
        or None to stop."""
        if stats is not None and (stats.numel() < 2 * len(PATH_NAMES) or
                                  stats.element_size() != 8 or not stats.is_contiguous()):
            raise ValueError("path stats need a contiguous 8-byte tensor of 2 * PATH_COUNT")
        _check(load().q3s_context_set_path_stats(self._h, None if stats is None
                                                 else stats.data_ptr()),
               "q3s_context_set_path_stats")

    def close(self) -> None:
        if self._h:
            load().q3s_context_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass


_default_ctx: dict = {}


def default_context(device: Optional[int] = None) -> Context:
    import torch
    d = torch.cuda.current_device() if device is None else int(device)
    if d not in _default_ctx:
        _default_ctx[d] = Context(d)
    return _default_ctx[d]


def make_params(n: int = 1, **fields) -> np.ndarray:
    """A q3s_row_params array; unspecified fields default to greedy-safe values."""
    p = np.zeros(n, dtype=ROW_PARAMS_DTYPE)
    p["temperature"] = 1.0
    p["top_p"] = 1.0
    p["repetition_penalty"] = 1.0
    p["suppress_from"] = NONE
    p["allow_token"] = NONE
    p["do_sample"] = 1
    for k, v in fields.items():
        p[k] = v
    return p


def _dptr(t) -> Optional[int]:
    return None if t is None else t.data_ptr()


def sample_batch(logits, params, seeds=None, subseqs=None, *, row_offsets=None, row_vocab=None,
                 vocab: Optional[int] = None, history=None, history_offsets=None,
                 uniform_override=None, debug: bool = False, ctx: Optional[Context] = None,
                 stream=None, out=None, history_ends=None):
    """One fused sampling launch over many rows (q3s_sample_batch).

    logits: CUDA tensor, float32 or bfloat16, either [R, V] (row stride taken
    from the tensor) or 1-D with row_offsets [R] (int64) and row_vocab [R]
    (int32).  params: CUDA uint8 tensor holding R (or 1, broadcast)
    q3s_row_params, or a numpy ROW_PARAMS_DTYPE array (copied to the device).
    seeds / subseqs: CUDA int64 tensors [R] (the u64 bit patterns).
    history: CUDA int16/uint16 tensor of concatenated ids with
    history_offsets [R+1] int64.  Returns (tokens int32 [R], status uint8 [R])
    and, with debug=True, also (probs [R, V] float32, masks [R, V] uint8).
    """
    return _launch_batch("q3s_sample_batch", logits, params, seeds, subseqs,
                         row_offsets=row_offsets, row_vocab=row_vocab, vocab=vocab,
                         history=history, history_offsets=history_offsets,
                         uniform_override=uniform_override, debug=debug, ctx=ctx, stream=stream,
                         out=out, history_ends=history_ends)


def sample_batch_static(logits, params, seeds=None, subseqs=None, *, row_offsets=None,
                        row_vocab=None, vocab: Optional[int] = None, history=None,
                        history_offsets=None, uniform_override=None, debug: bool = False,
                        ctx: Optional[Context] = None, stream=None, out=None,
                        history_ends=None):
    """sample_batch through q3s_sample_batch_static: the same launch with the
    library's file-scope device workspace, so the call itself allocates
    nothing on the device (pass `out` to keep torch from allocating the
    outputs).  Rejects vocab > MAX_VOCAB."""
    return _launch_batch("q3s_sample_batch_static", logits, params, seeds, subseqs,
                         row_offsets=row_offsets, row_vocab=row_vocab, vocab=vocab,
                         history=history, history_offsets=history_offsets,
                         uniform_override=uniform_override, debug=debug, ctx=ctx, stream=stream,
                         out=out, history_ends=history_ends)


class PreparedBatch:
    """A q3s_batch built once and launched many times (each launch is one C
    call: no argument marshalling per step).  Holds references to every
    tensor it points at; `tokens` / `status` are its outputs."""

    def __init__(self, entry: str, batch, ctx: "Context", keep: tuple, tokens, status):
        self._fn = getattr(load(), entry)
        self._entry = entry
        self._b = batch
        self._ref = ctypes.byref(batch)
        self._ctx = ctx
        self._keep = keep
        self.tokens = tokens
        self.status = status

    def __call__(self, stream: int) -> None:
        rc = self._fn(self._ctx.handle, self._ref, ctypes.c_void_p(stream))
        if rc != OK:
            _check(rc, self._entry)


def prepare_batch(logits, params, seeds=None, subseqs=None, *, row_offsets=None,
                  row_vocab=None, vocab: Optional[int] = None, history=None,
                  history_offsets=None, ctx: Optional[Context] = None, out=None,
                  static: bool = False, history_ends=None) -> PreparedBatch:
    """sample_batch's arguments fixed once; call the result with a stream
    handle to launch (q3s_sample_batch, or q3s_sample_batch_static)."""
    entry = "q3s_sample_batch_static" if static else "q3s_sample_batch"
    b, ctx, keep, tokens, status = _build_batch(
        logits, params, seeds, subseqs, row_offsets=row_offsets, row_vocab=row_vocab,
        vocab=vocab, history=history, history_offsets=history_offsets, uniform_override=None,
        debug=False, ctx=ctx, out=out, history_ends=history_ends)
    return PreparedBatch(entry, b, ctx, keep, tokens, status)


def _launch_batch(entry: str, logits, params, seeds, subseqs, *, row_offsets, row_vocab, vocab,
                  history, history_offsets, uniform_override, debug, ctx, stream, out,
                  history_ends=None):
    import torch
    b, ctx, keep, tokens, status = _build_batch(
        logits, params, seeds, subseqs, row_offsets=row_offsets, row_vocab=row_vocab,
        vocab=vocab, history=history, history_offsets=history_offsets,
        uniform_override=uniform_override, debug=debug, ctx=ctx, out=out,
        history_ends=history_ends)
    dev = logits.device
    s = torch.cuda.current_stream(dev).cuda_stream if stream is None else stream
    _check(getattr(load(), entry)(ctx.handle, ctypes.byref(b), ctypes.c_void_p(s)), entry)
    if debug:
        return tokens, status, keep[-2], keep[-1]
    return tokens, status


def _build_batch(logits, params, seeds, subseqs, *, row_offsets, row_vocab, vocab, history,
                 history_offsets, uniform_override, debug, ctx, out, history_ends=None):
    import torch
    dev = logits.device
    if logits.dtype == torch.float32:
        dt = DTYPE_F32
    elif logits.dtype == torch.bfloat16:
        dt = DTYPE_BF16
    else:
        raise TypeError("logits must be float32 or bfloat16")
    if logits.dim() == 2:
        R, V = logits.shape
        stride = logits.stride(0)
        if logits.stride(1) != 1:
            raise ValueError("logits rows must be contiguous")
    else:
        if row_offsets is None:
            raise ValueError("1-D logits need row_offsets")
        R = row_offsets.numel()
        stride = 0
        V = int(vocab if vocab is not None else int(row_vocab.max()))
    if vocab is not None:
        V = int(vocab)
    if isinstance(params, np.ndarray):
        params = torch.from_numpy(params.view(np.uint8).copy()).to(dev)
    nparams = params.numel() // ROW_PARAMS_DTYPE.itemsize
    if nparams not in (1, R):
        raise ValueError("params must hold 1 or R records")
    ctx = ctx or default_context(dev.index)
    if out is None:
        tokens = torch.empty(R, dtype=torch.int32, device=dev)
        status = torch.empty(R, dtype=torch.uint8, device=dev)
    else:
        tokens, status = out
    probs = masks = None
    if debug:
        probs = torch.empty((R, V), dtype=torch.float32, device=dev)
        masks = torch.empty((R, V), dtype=torch.uint8, device=dev)
    b = _Batch()
    b.logits = logits.data_ptr()
    b.dtype = dt
    b.vocab = V
    b.num_rows = R
    b.row_stride = stride
    b.row_offsets = _dptr(row_offsets)
    b.row_vocab = _dptr(row_vocab)
    b.params = params.data_ptr()
    b.params_stride = 0 if nparams == 1 else 1
    b.seeds = _dptr(seeds)
    b.subseqs = _dptr(subseqs)
    b.history = _dptr(history)
    b.history_offsets = _dptr(history_offsets)
    b.tokens = tokens.data_ptr()
    b.status = status.data_ptr()
    b.uniform_override = _dptr(uniform_override)
    b.probs = _dptr(probs)
    b.masks = _dptr(masks)
    b.probs_stride = V if debug else 0
    b.history_ends = _dptr(history_ends)
    keep = (logits, params, seeds, subseqs, row_offsets, row_vocab, history, history_offsets,
            history_ends, uniform_override, probs, masks)
    return b, ctx, keep, tokens, status


def embed_sum(codes, tables, text=None, *, ctx: Optional[Context] = None, stream=None,
              out=None):
    """The codebook embedding sum after sampling (q3s_embed_sum, talker.rs:568-580).

    codes: CUDA int32/uint32 tensor [R, G]; tables: G CUDA tensors [vocab_g, H]
    of one dtype (float32 or bfloat16); text: None, a [H] tensor (broadcast)
    or [R, H].  Returns (out [R, H] in the tables' dtype, status uint8 [R]);
    a row with a code outside its codebook has status STATUS_INVALID_CODE and
    zeros."""
    import torch
    if codes.dim() != 2:
        raise ValueError("codes must be [R, G]")
    if codes.dtype not in (torch.int32, torch.uint32):
        raise TypeError("codes must be int32 or uint32")
    R, G = codes.shape
    if len(tables) != G or G < 1 or G > MAX_CODE_GROUPS:
        raise ValueError("one table per code group (1..32)")
    dt = tables[0].dtype
    if dt == torch.float32:
        dcode = DTYPE_F32
    elif dt == torch.bfloat16:
        dcode = DTYPE_BF16
    else:
        raise TypeError("tables must be float32 or bfloat16")
    H = int(tables[0].shape[1])
    dev = codes.device
    # The C entry point has no sizes to check these against: a mismatch here
    # would make the kernel read or write past a buffer.
    for t in tables:
        if t.dtype != dt or t.dim() != 2 or int(t.shape[1]) != H or t.stride(1) != 1:
            raise ValueError("tables must share dtype and width and have contiguous rows")
        if t.stride(0) != H:
            raise ValueError("tables must be contiguous")
        if t.device != dev:
            raise ValueError("every table must be on the codes' device")
    codes = codes.contiguous()
    stride = 0
    if text is not None:
        if text.dtype != dt:
            raise TypeError("text must have the tables' dtype")
        if text.device != dev:
            raise ValueError("text must be on the codes' device")
        if text.dim() == 1:
            if int(text.shape[0]) != H or text.stride(0) != 1:
                raise ValueError("a 1-D text must be one contiguous row of H elements")
            stride = 0
        else:
            if text.dim() != 2 or text.shape[0] != R or int(text.shape[1]) != H or \
                    text.stride(1) != 1:
                raise ValueError("text must be [H] or [R, H] with contiguous rows")
            stride = text.stride(0)
    ctx = ctx or default_context(dev.index)
    if out is None:
        res = torch.empty((R, H), dtype=dt, device=dev)
        status = torch.empty(R, dtype=torch.uint8, device=dev)
    else:
        res, status = out
        if tuple(res.shape) != (R, H) or res.dtype != dt or res.device != dev or \
                not res.is_contiguous():
            raise ValueError("out[0] must be a contiguous [R, H] tensor of the tables' dtype "
                             "on the codes' device")
        if tuple(status.shape) != (R,) or status.dtype != torch.uint8 or status.device != dev:
            raise ValueError("out[1] must be a uint8 [R] tensor on the codes' device")
    ptrs = (ctypes.c_void_p * G)(*[t.data_ptr() for t in tables])
    vocab = (ctypes.c_int32 * G)(*[int(t.shape[0]) for t in tables])
    b = _EmbedBatch()
    b.dtype = dcode
    b.groups = G
    b.hidden = H
    b.num_rows = R
    b.codes = codes.data_ptr()
    b.tables = ctypes.cast(ptrs, ctypes.c_void_p)
    b.vocab = ctypes.cast(vocab, ctypes.c_void_p)
    b.text = _dptr(text)
    b.text_stride = stride
    b.out = res.data_ptr()
    b.status = status.data_ptr()
    s = torch.cuda.current_stream(dev).cuda_stream if stream is None else stream
    _check(load().q3s_embed_sum(ctx.handle, ctypes.byref(b), ctypes.c_void_p(s)), "q3s_embed_sum")
    return res, status


def greedy_batch(logits, suppress_from=None, allow_token=None, mode: int = GREEDY_SELECT,
                 ctx: Optional[Context] = None, stream=None):
    """Greedy argmax rows on device (q3s_greedy_batch); logits [R, V] CUDA."""
    import torch
    if logits.dim() == 1:
        logits = logits.view(1, -1)
    R, V = logits.shape
    dt = DTYPE_F32 if logits.dtype == torch.float32 else DTYPE_BF16
    ctx = ctx or default_context(logits.device.index)
    tokens = torch.empty(R, dtype=torch.int32, device=logits.device)
    status = torch.empty(R, dtype=torch.uint8, device=logits.device)
    s = torch.cuda.current_stream(logits.device).cuda_stream if stream is None else stream
    _check(load().q3s_greedy_batch(ctx.handle, ctypes.c_void_p(logits.data_ptr()), dt, R,
                                   logits.stride(0), V, _none(suppress_from), _none(allow_token),
                                   mode, ctypes.c_void_p(tokens.data_ptr()),
                                   ctypes.c_void_p(status.data_ptr()), ctypes.c_void_p(s)),
           "q3s_greedy_batch")
    return tokens, status


def greedy_select_on_device(logits, suppress_from=None, allow_token=None):
    """greedy_select_on_device (sampling.rs:72-117): a [1, 1] int32 device
    tensor; its value equals the vocabulary size when nothing is finite."""
    if logits.dim() == 2 and logits.shape[0] != 1:
        raise ValueError("greedy selection requires batch=1")
    if logits.numel() == 0:
        raise ValueError("greedy selection requires a non-empty vocabulary")
    tokens, _ = greedy_batch(logits.reshape(1, -1), suppress_from, allow_token, GREEDY_ON_DEVICE)
    return tokens.view(1, 1)


def greedy_select(logits, suppress_from=None, allow_token=None) -> int:
    """greedy_select (sampling.rs:40-60) on device; raises SamplingError."""
    tokens, status = greedy_batch(logits.reshape(1, -1), suppress_from, allow_token,
                                  GREEDY_SELECT)
    st = int(status.item())
    if st != STATUS_OK:
        raise SamplingError(st, status_message(st))
    return int(tokens.item())


class Sampler:
    """Sampler (sampling.rs:144-335) on the device: one Philox stream whose
    subsequence counter advances once per sampled call that drew."""

    def __init__(self, seed: int, ctx: Optional[Context] = None):
        self._ctx = ctx or default_context()
        self._h = ctypes.c_void_p()
        _check(load().q3s_sampler_create(self._ctx.handle, int(seed) & (2**64 - 1),
                                         ctypes.byref(self._h)), "q3s_sampler_create")

    def __del__(self):  # pragma: no cover
        try:
            if self._h:
                load().q3s_sampler_destroy(self._h)
        except Exception:
            pass

    def subsequence_counter(self) -> int:
        return int(load().q3s_sampler_subsequence_counter(self._h))

    def set_subsequence_counter(self, value: int) -> None:
        load().q3s_sampler_set_subsequence_counter(self._h, int(value) & (2**64 - 1))

    def diagnostics(self) -> dict:
        d = _Diagnostics()
        _check(load().q3s_sampler_get_diagnostics(self._h, ctypes.byref(d)),
               "q3s_sampler_get_diagnostics")
        n = int(d.sequence_len)
        return {"call_count": d.call_count, "sampled_calls": d.sampled_calls,
                "greedy_calls": d.greedy_calls,
                "history_nonempty_calls": d.history_nonempty_calls, "sequence_len": n,
                "sequence": list(d.sequence)[:n],
                "history_nonempty_sequence": list(d.history_nonempty_sequence)[:n]}

    def sample_with_mode_and_transfer_observer(
            self, logits, options: SamplingOptions, do_sample: bool, suppress_from=None,
            allow_token=None, history: Sequence[int] = (),
            observer: Optional[Callable[[int, int, int], None]] = None, stream=None) -> int:
        import torch
        if not logits.is_cuda:
            raise ValueError("logits must be a CUDA tensor")
        x = logits.reshape(-1)
        if not x.is_contiguous():
            x = x.contiguous()
        dt = DTYPE_F32 if x.dtype == torch.float32 else DTYPE_BF16
        if x.dtype not in (torch.float32, torch.bfloat16):
            raise TypeError("logits must be float32 or bfloat16")
        if isinstance(history, np.ndarray) and history.dtype == np.uint16 and \
                history.flags.c_contiguous:
            h = history
        else:
            h = np.ascontiguousarray(np.asarray(history, dtype=np.uint16))
        tok = ctypes.c_uint32(0)
        st = ctypes.c_int32(0)
        cb = TRANSFER_CALLBACK(0)
        if observer is not None:
            cb = TRANSFER_CALLBACK(lambda _u, direction, event, n: observer(direction, event, n))
        s = torch.cuda.current_stream(x.device).cuda_stream if stream is None else stream
        rc = load().q3s_sampler_sample_with_mode(
            self._h, ctypes.c_void_p(x.data_ptr() if x.numel() else 0), dt, x.numel(),
            ctypes.byref(options._c()), 1 if do_sample else 0, _none(suppress_from),
            _none(allow_token), h.ctypes.data_as(ctypes.c_void_p) if h.size else None, h.size,
            cb, None, ctypes.byref(tok), ctypes.byref(st), ctypes.c_void_p(s))
        if rc == E_SAMPLING:
            raise SamplingError(st.value, status_message(st.value))
        _check(rc, "q3s_sampler_sample_with_mode")
        return int(tok.value)

    def sample_with_mode(self, logits, options, do_sample, suppress_from=None, allow_token=None,
                         history=()) -> int:
        return self.sample_with_mode_and_transfer_observer(logits, options, do_sample,
                                                           suppress_from, allow_token, history)

    def sample_with_transfer_observer(self, logits, options, suppress_from=None,
                                      allow_token=None, history=(), observer=None) -> int:
        return self.sample_with_mode_and_transfer_observer(
            logits, options, options.temperature > 0.0, suppress_from, allow_token, history,
            observer)

    def sample(self, logits, options, suppress_from=None, allow_token=None, history=()) -> int:
        return self.sample_with_mode(logits, options, options.temperature > 0.0, suppress_from,
                                     allow_token, history)


def path_report(stats) -> dict:
    """{path name: {"rows", "cycles_per_row"}} of the paths a path-stats
    tensor saw (Context.set_path_stats)."""
    v = [int(x) for x in stats.cpu().tolist()]
    P = len(PATH_NAMES)
    return {name: {"rows": v[i], "cycles_per_row": v[P + i] / v[i]}
            for i, name in enumerate(PATH_NAMES) if v[i]}


def commit_rows(tokens, status, *, params=None, subseqs=None, codes=None, group: int = 0,
                frame_status=None, history=None, history_ends=None, history_limits=None,
                ctx: Optional[Context] = None, stream=None) -> None:
    """The device-side commit after a batched launch (q3s_commit_rows): the
    ids into column `group` of `codes` ([R, G] int32), the subsequence
    counters advanced on a draw, the first failure kept in `frame_status`
    (uint8 [R]) and, with `history`, the ids appended to each row's history
    range.  Every tensor is on the launch's device; nothing is copied."""
    import torch
    R = tokens.numel()
    c = _Commit()
    c.num_rows = R
    if params is not None and isinstance(params, np.ndarray):
        params = torch.from_numpy(params.view(np.uint8).copy()).to(tokens.device)
    c.params = _dptr(params)
    c.params_stride = 0 if params is None or params.numel() // ROW_PARAMS_DTYPE.itemsize == 1 \
        else 1
    c.tokens = tokens.data_ptr()
    c.status = status.data_ptr()
    c.subseqs = _dptr(subseqs)
    c.codes = _dptr(codes)
    c.codes_stride = codes.stride(0) if codes is not None else 0
    c.group = int(group)
    c.frame_status = _dptr(frame_status)
    c.history = _dptr(history)
    c.history_ends = _dptr(history_ends)
    c.history_limits = _dptr(history_limits)
    ctx = ctx or default_context(tokens.device.index)
    s = torch.cuda.current_stream(tokens.device).cuda_stream if stream is None else stream
    _check(load().q3s_commit_rows(ctx.handle, ctypes.byref(c), ctypes.c_void_p(s)),
           "q3s_commit_rows")


class Scheduler:
    """Continuous batching of sessions over the sampler (q3s_scheduler_*):
    each session keeps its own Philox stream, options and c0 history on the
    device; one frame samples every active session's talker row and code
    groups, one launch per step.  Joins and leaves take effect at
    begin_frame, which also retires sessions whose last frame failed."""

    def __init__(self, max_sessions: int, groups: int = 16, history_capacity: int = 4096,
                 ctx: Optional[Context] = None, device: int = 0):
        self.ctx = ctx or Context(device)
        self.groups = int(groups)
        self.max_sessions = int(max_sessions)
        self._h = ctypes.c_void_p()
        _check(load().q3s_scheduler_create(self.ctx.handle, self.max_sessions, self.groups,
                                           int(history_capacity), ctypes.byref(self._h)),
               "q3s_scheduler_create")
        self.active = []

    def add(self, session_id: int, seed: int, talker: SamplingOptions,
            predictor: SamplingOptions, *, talker_do_sample: bool = True,
            predictor_do_sample: bool = True, suppress_from=None, allow_token=None,
            history=(), subseq: int = 0) -> None:
        h = np.ascontiguousarray(np.asarray(history, dtype=np.uint16))
        c = _SessionConfig(int(session_id) & (2**64 - 1), int(seed) & (2**64 - 1),
                           int(subseq) & (2**64 - 1), talker._c(), predictor._c(),
                           1 if talker_do_sample else 0, 1 if predictor_do_sample else 0,
                           _none(suppress_from), _none(allow_token),
                           h.ctypes.data if h.size else None, h.size)
        _check(load().q3s_scheduler_add(self._h, ctypes.byref(c)), "q3s_scheduler_add")

    def cancel(self, session_id: int) -> None:
        _check(load().q3s_scheduler_cancel(self._h, int(session_id) & (2**64 - 1)),
               "q3s_scheduler_cancel")

    def begin_frame(self, stream=None) -> list:
        import torch
        ids = (ctypes.c_uint64 * self.max_sessions)()
        n = ctypes.c_int32(0)
        s = torch.cuda.current_stream(self.ctx.device).cuda_stream if stream is None else stream
        _check(load().q3s_scheduler_begin_frame(self._h, ids, self.max_sessions,
                                                ctypes.byref(n), ctypes.c_void_p(s)),
               "q3s_scheduler_begin_frame")
        self.active = list(ids[: n.value])
        return self.active

    def step(self, group: int, logits, stream=None) -> None:
        """logits: CUDA tensor [n, V] (float32 or bfloat16), row r for
        session active[r]."""
        import torch
        if logits.dtype == torch.float32:
            dt = DTYPE_F32
        elif logits.dtype == torch.bfloat16:
            dt = DTYPE_BF16
        else:
            raise TypeError("logits must be float32 or bfloat16")
        if logits.dim() != 2 or logits.stride(1) != 1 or logits.shape[0] != len(self.active):
            raise ValueError("logits must be [active sessions, vocab] with contiguous rows")
        s = torch.cuda.current_stream(self.ctx.device).cuda_stream if stream is None else stream
        _check(load().q3s_scheduler_step(self._h, int(group), logits.data_ptr(), dt,
                                         int(logits.shape[1]), logits.stride(0),
                                         ctypes.c_void_p(s)), "q3s_scheduler_step")

    def end_frame(self, stream=None):
        """(codes uint32 [n, groups], status uint8 [n]) of the frame."""
        import torch
        n = len(self.active)
        codes = np.zeros((n, self.groups), np.uint32)
        status = np.zeros(n, np.uint8)
        s = torch.cuda.current_stream(self.ctx.device).cuda_stream if stream is None else stream
        _check(load().q3s_scheduler_end_frame(self._h, codes.ctypes.data, status.ctypes.data,
                                              ctypes.c_void_p(s)), "q3s_scheduler_end_frame")
        return codes, status

    def codes_device(self):
        """The frame's codes as a CUDA int32 tensor [n, groups]: a view of
        the scheduler's device buffer (no copy), valid until the next
        begin_frame."""
        import torch
        n = len(self.active)
        ptr = load().q3s_scheduler_codes(self._h)

        class _View:
            __cuda_array_interface__ = {"shape": (n, self.groups), "typestr": "<i4",
                                        "data": (int(ptr), False), "version": 3}
        return torch.as_tensor(_View(), device=f"cuda:{self.ctx.device}")

    def session_state(self, session_id: int):
        """(subsequence counter, c0 history list) of an active session."""
        sub = ctypes.c_uint64(0)
        ln = ctypes.c_int64(0)
        _check(load().q3s_scheduler_session_state(self._h, int(session_id), ctypes.byref(sub),
                                                  ctypes.byref(ln), None, 0),
               "q3s_scheduler_session_state")
        h = np.zeros(max(ln.value, 1), np.uint16)
        _check(load().q3s_scheduler_session_state(self._h, int(session_id), ctypes.byref(sub),
                                                  ctypes.byref(ln), h.ctypes.data, h.size),
               "q3s_scheduler_session_state")
        return sub.value, h[: ln.value].tolist()

    def close(self) -> None:
        if self._h:
            load().q3s_scheduler_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass


def head_sample(hidden, weight, params, seeds=None, subseqs=None, *, history=None,
                history_offsets=None, history_ends=None, uniform_override=None,
                ctx: Optional[Context] = None, stream=None, out=None):
    """The head projection logits = hidden · weightᵀ and the sampling of its
    rows in one launch (q3s_head_sample).  hidden: CUDA [R, H] float32 or
    bfloat16 (R <= HEAD_MAX_ROWS, H a multiple of 8); weight: CUDA bfloat16
    [V, H], contiguous.  The sampling arguments are those of sample_batch.
    Returns (tokens int32 [R], status uint8 [R], logits float32 [R, V])."""
    import torch
    if hidden.dim() != 2 or hidden.stride(1) != 1:
        raise ValueError("hidden must be [R, H] with contiguous rows")
    if weight.dtype != torch.bfloat16 or weight.dim() != 2 or not weight.is_contiguous():
        raise ValueError("weight must be a contiguous bfloat16 [V, H] tensor")
    R, H = int(hidden.shape[0]), int(hidden.shape[1])
    V = int(weight.shape[0])
    if int(weight.shape[1]) != H:
        raise ValueError("weight and hidden disagree on H")
    if hidden.device != weight.device:
        raise ValueError("hidden and weight must be on one device")
    dev = hidden.device
    if hidden.dtype == torch.float32:
        hdt = DTYPE_F32
    elif hidden.dtype == torch.bfloat16:
        hdt = DTYPE_BF16
    else:
        raise TypeError("hidden must be float32 or bfloat16")
    if isinstance(params, np.ndarray):
        params = torch.from_numpy(params.view(np.uint8).copy()).to(dev)
    nparams = params.numel() // ROW_PARAMS_DTYPE.itemsize
    if nparams not in (1, R):
        raise ValueError("params must hold 1 or R records")
    ctx = ctx or default_context(dev.index)
    if out is None:
        tokens = torch.empty(R, dtype=torch.int32, device=dev)
        status = torch.empty(R, dtype=torch.uint8, device=dev)
        logits = torch.empty((R, V), dtype=torch.float32, device=dev)
    else:
        tokens, status, logits = out
    hb = _HeadBatch()
    hb.hidden = hidden.data_ptr()
    hb.hidden_dtype = hdt
    hb.hidden_size = H
    hb.hidden_stride = hidden.stride(0)
    hb.weight = weight.data_ptr()
    hb.logits = logits.data_ptr()
    b = hb.sample
    b.vocab = V
    b.num_rows = R
    b.params = params.data_ptr()
    b.params_stride = 0 if nparams == 1 else 1
    b.seeds = _dptr(seeds)
    b.subseqs = _dptr(subseqs)
    b.history = _dptr(history)
    b.history_offsets = _dptr(history_offsets)
    b.history_ends = _dptr(history_ends)
    b.tokens = tokens.data_ptr()
    b.status = status.data_ptr()
    b.uniform_override = _dptr(uniform_override)
    s = torch.cuda.current_stream(dev).cuda_stream if stream is None else stream
    _check(load().q3s_head_sample(ctx.handle, ctypes.byref(hb), ctypes.c_void_p(s)),
           "q3s_head_sample")
    return tokens, status, logits


def sample_commit(logits, params, seeds, subseqs, *, codes=None, group: int = 0,
                  frame_status=None, commit_history=None, history_limits=None, row_offsets=None,
                  row_vocab=None, vocab: Optional[int] = None, history=None, history_offsets=None,
                  history_ends=None, ctx: Optional[Context] = None, stream=None, out=None):
    """sample_batch and commit_rows in one launch (q3s_sample_commit): each
    row's warp commits the row after storing its result.  commit_history:
    the history array to append the ids to (normally `history`), with
    history_ends / history_limits; subseqs are advanced in place."""
    import torch
    b, ctx, keep, tokens, status = _build_batch(
        logits, params, seeds, subseqs, row_offsets=row_offsets, row_vocab=row_vocab,
        vocab=vocab, history=history, history_offsets=history_offsets, uniform_override=None,
        debug=False, ctx=ctx, out=out, history_ends=history_ends)
    c = _Commit()
    c.subseqs = _dptr(subseqs)
    c.codes = _dptr(codes)
    c.codes_stride = codes.stride(0) if codes is not None else 0
    c.group = int(group)
    c.frame_status = _dptr(frame_status)
    c.history = _dptr(commit_history)
    c.history_ends = _dptr(history_ends) if commit_history is not None else None
    c.history_limits = _dptr(history_limits)
    dev = logits.device
    s = torch.cuda.current_stream(dev).cuda_stream if stream is None else stream
    _check(load().q3s_sample_commit(ctx.handle, ctypes.byref(b), ctypes.byref(c),
                                    ctypes.c_void_p(s)), "q3s_sample_commit")
    return tokens, status
