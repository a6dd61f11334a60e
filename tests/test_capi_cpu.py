"""C ABI checks that need no GPU: the library builds and loads, exports every
symbol include/q3s_sampler.h declares, its struct layouts match the Python
binding, and its status messages are the reference's error strings."""
import re
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

import q3s

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "q3s_sampler.h"


def declared_functions() -> set:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = set(re.findall(r"^[A-Za-z_][\w\s\*]*?\b(q3s_\w+)\s*\(", text, flags=re.M))
    return {n for n in names if not n.startswith("q3s_transfer_callback")}


def test_library_loads_and_exports_every_declared_symbol():
    lib = q3s.load()
    declared = declared_functions()
    assert declared == set(q3s.EXPORTED_SYMBOLS)
    for name in declared:
        assert hasattr(lib, name), name
    nm = shutil.which("nm")
    if nm:
        out = subprocess.run([nm, "-D", "--defined-only", str(q3s.LIB_PATH)], capture_output=True,
                             text=True, check=True).stdout
        exported = set(re.findall(r"\bT (q3s_\w+)$", out, flags=re.M))
        assert declared <= exported


def test_abi_version_and_status_messages():
    lib = q3s.load()
    assert lib.q3s_abi_version() == 2
    # The reference's error strings (src/talker/sampling.rs:281-296, 642-650,
    # 675-678, 705-718, 58-59).
    expect = {
        q3s.STATUS_INVALID_REPETITION_PENALTY:
            "invalid repetition_penalty: expected finite value > 0.0",
        q3s.STATUS_INVALID_TEMPERATURE:
            "invalid temperature: expected finite value > 0.0 when sampling is enabled",
        q3s.STATUS_INVALID_TOP_P: "invalid top_p: expected finite value in (0.0, 1.0]",
        q3s.STATUS_SUPPRESSION_NO_CANDIDATE: "suppression left no finite candidate",
        q3s.STATUS_NO_CANDIDATE: "no finite sampling candidate",
        q3s.STATUS_INVALID_DENOMINATOR: "invalid softmax denominator",
        q3s.STATUS_INVALID_CODE: "embedding code outside its codebook",
        q3s.STATUS_HISTORY_FULL: "c0 history capacity exhausted",
    }
    for st, msg in expect.items():
        assert q3s.status_message(st) == msg


def test_struct_layouts_match_binding(tmp_path):
    gcc = shutil.which("gcc")
    if not gcc:
        pytest.skip("no C compiler")
    src = tmp_path / "layout.c"
    src.write_text(r'''
#include <stddef.h>
#include <stdio.h>
#include "q3s_sampler.h"
int main(void) {
  printf("%zu %zu %zu %zu %zu %zu %zu %zu %zu %zu %zu %zu %zu %zu %zu %zu %zu %zu %zu\n", sizeof(q3s_row_params),
         offsetof(q3s_row_params, top_k), offsetof(q3s_row_params, do_sample),
         offsetof(q3s_row_params, suppress_from), offsetof(q3s_row_params, allow_token),
         offsetof(q3s_row_params, ctr_lo), sizeof(q3s_batch), offsetof(q3s_batch, probs_stride),
         sizeof(q3s_sampling_options), sizeof(q3s_sampler_diagnostics),
         sizeof(q3s_embed_batch), offsetof(q3s_embed_batch, text_stride),
         offsetof(q3s_embed_batch, status), offsetof(q3s_batch, history_ends),
         sizeof(q3s_commit), offsetof(q3s_commit, group), offsetof(q3s_commit, history_limits),
         sizeof(q3s_head_batch), offsetof(q3s_head_batch, sample));
  return 0;
}
''')
    exe = tmp_path / "layout"
    subprocess.run([gcc, "-I", str(ROOT / "include"), "-o", str(exe), str(src)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True,
                                          check=True).stdout.split()]
    dt = q3s.ROW_PARAMS_DTYPE
    import ctypes
    assert got == [dt.itemsize, dt.fields["top_k"][1], dt.fields["do_sample"][1],
                   dt.fields["suppress_from"][1], dt.fields["allow_token"][1],
                   dt.fields["ctr_lo"][1], ctypes.sizeof(q3s._Batch),
                   q3s._Batch.probs_stride.offset, ctypes.sizeof(q3s._Options),
                   ctypes.sizeof(q3s._Diagnostics), ctypes.sizeof(q3s._EmbedBatch),
                   q3s._EmbedBatch.text_stride.offset, q3s._EmbedBatch.status.offset,
                   q3s._Batch.history_ends.offset, ctypes.sizeof(q3s._Commit),
                   q3s._Commit.group.offset, q3s._Commit.history_limits.offset,
                   ctypes.sizeof(q3s._HeadBatch), q3s._HeadBatch.sample.offset]


def test_context_without_device_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(q3s.LibraryError):
        q3s.Context(0)


def test_make_params_defaults():
    p = q3s.make_params(3, top_k=50)
    assert p.dtype == q3s.ROW_PARAMS_DTYPE and p.size == 3
    assert (p["suppress_from"] == -1).all() and (p["top_k"] == 50).all()
    assert np.all(p["do_sample"] == 1)
