"""Seeded synthetic sampling workloads with the shapes and distributions of the
reference's five sampling configurations (there is no dataset: the sampler
consumes logits, and every configuration states their distribution).

    talker_single   1 row x 3072 f32 ~ N(0, 2.5^2) per step; 256-id history in
                    [0, 2048); rp 1.05, T 0.9, k 50, p 1.0; ids [2048, 3072)
                    suppressed except EOS 2150; Philox seed 42, subseq = step
    cp_frame        64 streams x 15 groups of bf16 [64, 2048] ~ N(0, 3^2);
                    T 0.9, k 50, p 1.0, no penalty or suppression; seeds 0..63,
                    subseq = group
    talker_batch    1024 x 3072 f32 ~ N(0, 2^2) plus +8 on 5 positions per
                    row; history length U{0..4096}, ids in [0, 2048); rp 1.1,
                    T 0.7, k off, p 0.8; suppression as talker_single
    bandwidth       65536 x 3072 f32 ~ N(0, 1); k in {1, 50, 256}, p 1.0,
                    T 1.0, no penalty
    hetero          4096 streams x (1 talker row of 3072 + 15 code-predictor
                    rows of 2048), f32 Gumbel(0, 1) + N(0, 1.5^2); per row
                    T ~ U[0.5, 1.2], k ~ U{1..200}, p ~ U[0.5, 1.0],
                    rp ~ U[1.0, 1.3], history 0..2048 ids; talker rows keep the
                    talker suppression

Generators run on the CPU with numpy (small cases, bit-reproducible) or on
the device with torch (full sizes).  All arrays are returned as torch tensors
on the requested device, plus the host copies the oracle needs.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np

from . import ROW_PARAMS_DTYPE, NONE, make_params

TALKER_V = 3072
CP_V = 2048
TALKER_SUPPRESS_FROM = 2048
TALKER_EOS = 2150


@dataclass
class Workload:
    name: str
    logits: object                    # torch tensor [R, V] or 1-D with row_offsets
    params: np.ndarray                # ROW_PARAMS_DTYPE [R] or [1]
    seeds: np.ndarray                 # uint64 [R]
    subseqs: np.ndarray               # uint64 [R]
    vocab: int
    row_offsets: Optional[np.ndarray] = None   # int64 [R]
    row_vocab: Optional[np.ndarray] = None     # int32 [R]
    history: Optional[np.ndarray] = None       # uint16
    history_offsets: Optional[np.ndarray] = None  # int64 [R+1]
    meta: dict = field(default_factory=dict)

    @property
    def num_rows(self) -> int:
        return int(self.seeds.size)

    def device_args(self, device):
        """Tensors for q3s.sample_batch on `device`."""
        import torch

        def t(a, dt=None):
            if a is None:
                return None
            x = torch.from_numpy(np.ascontiguousarray(a))
            if dt is not None:
                x = x.view(dt)
            return x.to(device)
        args = {
            "params": t(self.params.view(np.uint8)),
            "seeds": t(self.seeds.view(np.int64)),
            "subseqs": t(self.subseqs.view(np.int64)),
            "row_offsets": t(self.row_offsets),
            "row_vocab": t(self.row_vocab),
            "history": t(None if self.history is None else self.history.view(np.int16)),
            "history_offsets": t(self.history_offsets),
        }
        if self.row_offsets is not None:
            args["vocab"] = self.vocab
        return args

    def host_logits(self, rows=None) -> np.ndarray:
        """Flat f32 host copy of the logits (of `rows` when given, re-based)."""
        import torch
        x = self.logits
        if rows is None:
            return x.float().reshape(-1).cpu().numpy()
        if self.row_offsets is None:
            return x[torch.as_tensor(rows, device=x.device)].float().reshape(-1).cpu().numpy()
        flat = x.float().reshape(-1)
        parts = [flat[int(self.row_offsets[r]): int(self.row_offsets[r]) + int(self.row_vocab[r])]
                 for r in rows]
        return torch.cat(parts).cpu().numpy()

    def oracle_layout(self, rows=None):
        """(logits, offsets, vocab, params, seeds, subseqs, history, hoff) for
        oracle.sample_rows over `rows` (all rows when None)."""
        R = self.num_rows
        rows = np.arange(R) if rows is None else np.asarray(rows)
        logits = self.host_logits(rows)
        if self.row_vocab is not None:
            vocab = self.row_vocab[rows].astype(np.int32)
        else:
            vocab = np.full(rows.size, self.vocab, np.int32)
        offsets = np.zeros(rows.size, np.int64)
        offsets[1:] = np.cumsum(vocab[:-1].astype(np.int64))
        params = self.params[rows] if self.params.size > 1 else self.params
        hist = hoff = None
        if self.history_offsets is not None:
            chunks = [self.history[self.history_offsets[r]:self.history_offsets[r + 1]]
                      for r in rows]
            hoff = np.zeros(rows.size + 1, np.int64)
            hoff[1:] = np.cumsum([c.size for c in chunks])
            hist = np.concatenate(chunks) if chunks else np.zeros(0, np.uint16)
        return (logits, offsets, vocab, params, self.seeds[rows], self.subseqs[rows], hist, hoff)


def _to_device(arr: np.ndarray, device, dtype=None):
    import torch
    x = torch.from_numpy(arr)
    if dtype is not None:
        x = x.to(dtype)
    return x.to(device)


def _normal(rng, shape, scale, device, gen_seed: int):
    """N(0, scale^2) f32 logits: numpy on CPU, torch's generator on CUDA."""
    import torch
    dev = torch.device(device)
    if dev.type == "cuda":
        g = torch.Generator(device=dev)
        g.manual_seed(gen_seed)
        return torch.randn(shape, generator=g, device=dev, dtype=torch.float32) * scale
    return torch.from_numpy((rng.standard_normal(shape, dtype=np.float32) * np.float32(scale)))


def talker_single(device="cpu", steps: int = 1000, seed: int = 0) -> Workload:
    rng = np.random.default_rng(seed)
    logits = _normal(rng, (steps, TALKER_V), 2.5, device, seed)
    hist_one = rng.integers(0, 2048, 256).astype(np.uint16)
    history = np.tile(hist_one, steps)
    hoff = np.arange(steps + 1, dtype=np.int64) * 256
    params = make_params(1, temperature=0.9, top_k=50, top_p=1.0, repetition_penalty=1.05,
                         suppress_from=TALKER_SUPPRESS_FROM, allow_token=TALKER_EOS)
    return Workload("talker_single", logits.to(device), params,
                    np.full(steps, 42, np.uint64), np.arange(steps, dtype=np.uint64), TALKER_V,
                    history=history, history_offsets=hoff,
                    meta={"steps": steps, "rows_per_step": 1})


def cp_frame(device="cpu", streams: int = 64, groups: int = 15, seed: int = 1) -> Workload:
    import torch
    rng = np.random.default_rng(seed)
    x = _normal(rng, (groups * streams, CP_V), 3.0, device, seed)
    logits = x.to(torch.bfloat16).to(device)
    params = make_params(1, temperature=0.9, top_k=50, top_p=1.0, repetition_penalty=1.0)
    seeds = np.tile(np.arange(streams, dtype=np.uint64), groups)
    subseqs = np.repeat(np.arange(groups, dtype=np.uint64), streams)
    return Workload("cp_frame", logits, params, seeds, subseqs, CP_V,
                    meta={"streams": streams, "groups": groups})


def talker_batch(device="cpu", rows: int = 1024, seed: int = 2) -> Workload:
    import torch
    rng = np.random.default_rng(seed)
    x = _normal(rng, (rows, TALKER_V), 2.0, device, seed)
    spikes = rng.integers(0, TALKER_V, (rows, 5))
    add = torch.zeros((rows, TALKER_V), dtype=torch.float32)
    add.scatter_(1, torch.from_numpy(spikes), 8.0)
    logits = (x.to(device) + add.to(device)).contiguous()
    lens = rng.integers(0, 4097, rows)
    hoff = np.zeros(rows + 1, np.int64)
    hoff[1:] = np.cumsum(lens)
    history = rng.integers(0, 2048, int(hoff[-1])).astype(np.uint16)
    params = make_params(1, temperature=0.7, top_k=0, top_p=0.8, repetition_penalty=1.1,
                         suppress_from=TALKER_SUPPRESS_FROM, allow_token=TALKER_EOS)
    seeds = rng.integers(0, 2**63, rows).astype(np.uint64)
    subseqs = rng.integers(0, 1000, rows).astype(np.uint64)
    return Workload("talker_batch", logits, params, seeds, subseqs, TALKER_V, history=history,
                    history_offsets=hoff)


def bandwidth(device="cpu", rows: int = 65536, top_k: int = 50, seed: int = 3) -> Workload:
    rng = np.random.default_rng(seed)
    logits = _normal(rng, (rows, TALKER_V), 1.0, device, seed).to(device)
    params = make_params(1, temperature=1.0, top_k=top_k, top_p=1.0, repetition_penalty=1.0)
    seeds = np.arange(rows, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15)
    subseqs = np.zeros(rows, np.uint64)
    return Workload("bandwidth", logits, params, seeds, subseqs, TALKER_V,
                    meta={"top_k": top_k})


def hetero(device="cpu", streams: int = 4096, seed: int = 4) -> Workload:
    import torch
    rng = np.random.default_rng(seed)
    per = TALKER_V + 15 * CP_V
    total = streams * per
    dev = torch.device(device)
    if dev.type == "cuda":
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        u = torch.rand(total, generator=g, device=dev, dtype=torch.float32)
        u = u.clamp_(min=1e-12)
        gumbel = -torch.log(-torch.log(u))
        logits = gumbel + 1.5 * torch.randn(total, generator=g, device=dev, dtype=torch.float32)
    else:
        u = rng.random(total, dtype=np.float32).clip(1e-12, None)
        logits = torch.from_numpy(-np.log(-np.log(u)).astype(np.float32) +
                                  rng.standard_normal(total, dtype=np.float32) * np.float32(1.5))
    R = streams * 16
    row_vocab = np.tile(np.array([TALKER_V] + [CP_V] * 15, np.int32), streams)
    row_offsets = np.zeros(R, np.int64)
    row_offsets[1:] = np.cumsum(row_vocab[:-1].astype(np.int64))
    params = np.zeros(R, dtype=ROW_PARAMS_DTYPE)
    params["temperature"] = rng.uniform(0.5, 1.2, R)
    params["top_k"] = rng.integers(1, 201, R)
    params["top_p"] = rng.uniform(0.5, 1.0, R)
    params["repetition_penalty"] = rng.uniform(1.0, 1.3, R)
    params["do_sample"] = 1
    talker = (np.arange(R) % 16) == 0
    params["suppress_from"] = np.where(talker, TALKER_SUPPRESS_FROM, NONE)
    params["allow_token"] = np.where(talker, TALKER_EOS, NONE)
    lens = rng.integers(0, 2049, R)
    hoff = np.zeros(R + 1, np.int64)
    hoff[1:] = np.cumsum(lens)
    history = rng.integers(0, 2048, int(hoff[-1])).astype(np.uint16)
    seeds = np.repeat(rng.integers(0, 2**63, streams).astype(np.uint64), 16)
    subseqs = np.tile(np.arange(16, dtype=np.uint64), streams)
    return Workload("hetero", logits.to(device), params, seeds, subseqs, TALKER_V,
                    row_offsets=row_offsets, row_vocab=row_vocab, history=history,
                    history_offsets=hoff, meta={"streams": streams})


WORKLOADS = {
    "talker_single": talker_single,
    "cp_frame": cp_frame,
    "talker_batch": talker_batch,
    "bandwidth": bandwidth,
    "hetero": hetero,
}
