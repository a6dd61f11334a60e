"""ORACLE — test infrastructure only.

ctypes binding of oracle/libq3s_oracle.so, the CPU restatement of the
reference sampler (qwen3tts-rs src/talker/sampling.rs).  Imported only by
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg, always as the
checker, never as the thing measured for the product.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libq3s_oracle.so"

EXP_CR = 0
EXP_LIBM = 1

OK = 0
INVALID_REPETITION_PENALTY = 1
INVALID_TEMPERATURE = 2
INVALID_TOP_P = 3
SUPPRESSION_NO_CANDIDATE = 4
NO_CANDIDATE = 5
INVALID_DENOMINATOR = 6

# Same layout as q3s_row_params in include/q3s_sampler.h (48 bytes).
ROW_PARAMS_DTYPE = np.dtype([
    ("temperature", "<f8"), ("top_p", "<f8"), ("repetition_penalty", "<f8"),
    ("top_k", "<u4"), ("do_sample", "<u4"), ("suppress_from", "<i4"),
    ("allow_token", "<i4"), ("ctr_lo", "<u4"), ("reserved", "<u4"),
])
assert ROW_PARAMS_DTYPE.itemsize == 48


class _Options(ctypes.Structure):
    _fields_ = [("temperature", ctypes.c_double), ("top_k", ctypes.c_uint64),
                ("top_p", ctypes.c_double), ("repetition_penalty", ctypes.c_double)]


class _Trace(ctypes.Structure):
    _fields_ = [("after_penalty", ctypes.c_void_p), ("after_temperature", ctypes.c_void_p),
                ("final_probs", ctypes.c_void_p), ("masks", ctypes.c_void_p),
                ("topk_threshold", ctypes.c_float), ("draw_threshold", ctypes.c_float),
                ("draw_sum", ctypes.c_float), ("boundary_gap", ctypes.c_double),
                ("topp_gap", ctypes.c_double)]


class _Sampler(ctypes.Structure):
    _fields_ = [("seed", ctypes.c_uint64), ("subseq_counter", ctypes.c_uint64),
                ("ctr_lo", ctypes.c_uint32), ("call_count", ctypes.c_uint32),
                ("sampled_calls", ctypes.c_uint32), ("greedy_calls", ctypes.c_uint32),
                ("history_nonempty_calls", ctypes.c_uint32),
                ("history_nonempty_sequence", ctypes.c_uint8 * 64),
                ("sequence", ctypes.c_uint8 * 64), ("sequence_len", ctypes.c_uint64)]


_lib = None


def build() -> Path:
    """Compile the oracle with its Makefile (g++ -O3 -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", str(HERE), str(LIB_PATH)], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        L.q3o_cr_expf.restype = ctypes.c_float
        L.q3o_cr_expf.argtypes = [ctypes.c_float]
        L.q3o_expf.restype = ctypes.c_float
        L.q3o_expf.argtypes = [ctypes.c_float, ctypes.c_int]
        L.q3o_philox4x32_10.argtypes = [ctypes.POINTER(ctypes.c_uint32), ctypes.c_uint32,
                                        ctypes.c_uint32, ctypes.POINTER(ctypes.c_uint32)]
        L.q3o_next_uniform.restype = ctypes.c_float
        L.q3o_next_uniform.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint32]
        L.q3o_apply_repetition_penalty.argtypes = [ctypes.c_void_p, ctypes.c_size_t,
                                                   ctypes.c_void_p, ctypes.c_size_t,
                                                   ctypes.c_double]
        L.q3o_sample_logits.restype = ctypes.c_int
        L.q3o_sample_logits.argtypes = [
            ctypes.c_void_p, ctypes.c_size_t, _Options, ctypes.c_int64, ctypes.c_int64,
            ctypes.c_void_p, ctypes.c_size_t, ctypes.c_float, ctypes.c_int,
            ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_int),
            ctypes.POINTER(_Trace)]
        L.q3o_greedy_select.restype = ctypes.c_int
        L.q3o_greedy_select.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int64,
                                        ctypes.c_int64, ctypes.POINTER(ctypes.c_uint32)]
        L.q3o_greedy_select_on_device.restype = ctypes.c_uint32
        L.q3o_greedy_select_on_device.argtypes = [ctypes.c_void_p, ctypes.c_size_t,
                                                  ctypes.c_int64, ctypes.c_int64]
        L.q3o_sampler_init.argtypes = [ctypes.POINTER(_Sampler), ctypes.c_uint64]
        L.q3o_sampler_sample_with_mode.restype = ctypes.c_int
        L.q3o_sampler_sample_with_mode.argtypes = [
            ctypes.POINTER(_Sampler), ctypes.c_void_p, ctypes.c_size_t, _Options, ctypes.c_int,
            ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int,
            ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(_Trace)]
        L.q3o_sample_rows_ex.restype = ctypes.c_int
        L.q3o_sample_rows_ex.argtypes = [
            ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _opt(o) -> _Options:
    return _Options(float(o["temperature"]), int(o["top_k"]), float(o["top_p"]),
                    float(o["repetition_penalty"]))


def _none(v) -> int:
    return -1 if v is None else int(v)


def cr_expf(x: float) -> float:
    return lib().q3o_cr_expf(x)


def expf(x: float, exp_mode: int = EXP_CR) -> float:
    return lib().q3o_expf(x, exp_mode)


def philox4x32_10(ctr, seed_lo: int, seed_hi: int) -> list[int]:
    c = (ctypes.c_uint32 * 4)(*[int(v) & 0xFFFFFFFF for v in ctr])
    out = (ctypes.c_uint32 * 4)()
    lib().q3o_philox4x32_10(c, seed_lo & 0xFFFFFFFF, seed_hi & 0xFFFFFFFF, out)
    return list(out)


def next_uniform(seed: int, subsequence: int, ctr_lo: int = 0) -> float:
    return lib().q3o_next_uniform(seed & (2**64 - 1), subsequence & (2**64 - 1), ctr_lo)


def apply_repetition_penalty(logits, history, penalty: float) -> np.ndarray:
    x = np.array(logits, dtype=np.float32)
    h = np.array(history, dtype=np.uint16)
    lib().q3o_apply_repetition_penalty(_ptr(x), x.size, _ptr(h), h.size, float(penalty))
    return x


@dataclass
class SampleResult:
    status: int
    token: int
    drew: bool
    after_penalty: np.ndarray
    after_temperature: np.ndarray
    final_probs: np.ndarray
    masks: np.ndarray
    topk_threshold: float
    draw_threshold: float
    draw_sum: float
    boundary_gap: float
    topp_gap: float


def sample_logits(logits, options, suppress_from=None, allow_token=None, history=(),
                  uniform: float = 0.5, exp_mode: int = EXP_CR) -> SampleResult:
    """sample_logits_with_scratch (sampling.rs:561-730) with a fixed draw."""
    x = np.ascontiguousarray(logits, dtype=np.float32)
    n = x.size
    h = np.array(history, dtype=np.uint16)
    ap = np.zeros(n, np.float32)
    at = np.zeros(n, np.float32)
    fp = np.zeros(n, np.float32)
    mk = np.zeros(n, np.uint8)
    tr = _Trace(_ptr(ap).value, _ptr(at).value, _ptr(fp).value, _ptr(mk).value, 0.0, 0.0, 0.0,
                float("inf"), float("inf"))
    tok = ctypes.c_uint32(0)
    drew = ctypes.c_int(0)
    st = lib().q3o_sample_logits(_ptr(x), n, _opt(options), _none(suppress_from),
                                 _none(allow_token), _ptr(h), h.size, float(uniform), exp_mode,
                                 ctypes.byref(tok), ctypes.byref(drew), ctypes.byref(tr))
    return SampleResult(st, tok.value, bool(drew.value), ap, at, fp, mk, tr.topk_threshold,
                        tr.draw_threshold, tr.draw_sum, tr.boundary_gap, tr.topp_gap)


def greedy_select(logits, suppress_from=None, allow_token=None):
    x = np.ascontiguousarray(logits, dtype=np.float32)
    tok = ctypes.c_uint32(0)
    st = lib().q3o_greedy_select(_ptr(x), x.size, _none(suppress_from), _none(allow_token),
                                 ctypes.byref(tok))
    return st, tok.value


def greedy_select_on_device(logits, suppress_from=None, allow_token=None) -> int:
    x = np.ascontiguousarray(logits, dtype=np.float32)
    return lib().q3o_greedy_select_on_device(_ptr(x), x.size, _none(suppress_from),
                                             _none(allow_token))


class OracleSampler:
    """Sampler (sampling.rs:144-335) over the CPU restatement."""

    def __init__(self, seed: int, exp_mode: int = EXP_CR):
        self._s = _Sampler()
        self.exp_mode = exp_mode
        lib().q3o_sampler_init(ctypes.byref(self._s), seed & (2**64 - 1))

    @property
    def subsequence_counter(self) -> int:
        return self._s.subseq_counter

    @subsequence_counter.setter
    def subsequence_counter(self, v: int) -> None:
        self._s.subseq_counter = v & (2**64 - 1)

    def diagnostics(self) -> dict:
        s = self._s
        return {"call_count": s.call_count, "sampled_calls": s.sampled_calls,
                "greedy_calls": s.greedy_calls,
                "history_nonempty_calls": s.history_nonempty_calls,
                "sequence_len": s.sequence_len,
                "sequence": list(s.sequence)[: s.sequence_len],
                "history_nonempty_sequence": list(s.history_nonempty_sequence)[: s.sequence_len]}

    def sample_with_mode(self, logits, options, do_sample: bool, suppress_from=None,
                         allow_token=None, history=()):
        x = np.ascontiguousarray(logits, dtype=np.float32)
        h = np.array(history, dtype=np.uint16)
        tok = ctypes.c_uint32(0)
        st = lib().q3o_sampler_sample_with_mode(
            ctypes.byref(self._s), _ptr(x), x.size, _opt(options), 1 if do_sample else 0,
            _none(suppress_from), _none(allow_token), _ptr(h), h.size, self.exp_mode,
            ctypes.byref(tok), None)
        return st, tok.value

    def sample(self, logits, options, suppress_from=None, allow_token=None, history=()):
        return self.sample_with_mode(logits, options, options["temperature"] > 0.0,
                                     suppress_from, allow_token, history)


def sample_rows(logits: np.ndarray, offsets: np.ndarray, vocab: np.ndarray, params: np.ndarray,
                seeds: np.ndarray, subseqs: np.ndarray, history: np.ndarray | None = None,
                history_offsets: np.ndarray | None = None, uniform_override=None,
                exp_mode: int = EXP_CR, want_probs: bool = False, nthreads: int = 1):
    """One batched call over rows laid out like q3s_batch (host arrays)."""
    R = int(offsets.size)
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    offsets = np.ascontiguousarray(offsets, dtype=np.int64)
    vocab = np.ascontiguousarray(vocab, dtype=np.int32)
    params = np.ascontiguousarray(params, dtype=ROW_PARAMS_DTYPE)
    pstride = 0 if params.size == 1 else 1
    seeds = np.ascontiguousarray(seeds, dtype=np.uint64)
    subseqs = np.ascontiguousarray(subseqs, dtype=np.uint64)
    if history is not None:
        history = np.ascontiguousarray(history, dtype=np.uint16)
        history_offsets = np.ascontiguousarray(history_offsets, dtype=np.int64)
    uo = None if uniform_override is None else np.ascontiguousarray(uniform_override, np.float32)
    tokens = np.zeros(R, np.uint32)
    status = np.zeros(R, np.uint8)
    gap = np.zeros(R, np.float64)
    tgap = np.zeros(R, np.float64)
    stride = int(vocab.max()) if (want_probs and R) else 0
    probs = np.zeros(R * stride, np.float32) if want_probs else None
    masks = np.zeros(R * stride, np.uint8) if want_probs else None
    lib().q3o_sample_rows_ex(_ptr(logits), R, _ptr(offsets), _ptr(vocab), _ptr(params),
                             pstride, _ptr(seeds), _ptr(subseqs), _ptr(history),
                             _ptr(history_offsets), _ptr(uo), exp_mode, _ptr(tokens),
                             _ptr(status), _ptr(probs), _ptr(masks), stride, _ptr(gap),
                             _ptr(tgap), int(nthreads))
    out = {"tokens": tokens, "status": status, "boundary_gap": gap, "topp_gap": tgap}
    if want_probs:
        out["probs"] = probs.reshape(R, stride)
        out["masks"] = masks.reshape(R, stride)
    return out


def cpu_count() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1
