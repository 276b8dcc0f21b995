"""The C ABI (include/chia_attn.h) without a GPU: exports, struct layout,
argument validation (every error is reported before anything is launched)."""

import ctypes
import os
import re
import shutil
import subprocess

import pytest

from chia_proj_b200 import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "chia_attn.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"CHIA_API\s+[\w\s\*]*?\b(chia_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol(lib):
    decl = declared_symbols()
    assert decl, "no CHIA_API declarations found"
    assert set(decl) == set(N.EXPORTED_SYMBOLS)
    for name in decl:
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", N.LIB_PATH], capture_output=True,
                         text=True).stdout
    exported = set(re.findall(r"\b(chia_\w+)\b", out))
    assert set(decl) <= exported


def test_abi_version_and_status_strings(lib):
    assert lib.chia_attn_abi_version() == N.ABI_VERSION
    for code, name in N.STATUS.items():
        s = lib.chia_attn_status_string(code).decode()
        assert s and s != "unknown status"
    assert lib.chia_attn_status_string(99) == b"unknown status"


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_struct_layout_matches_header(tmp_path):
    fields = [f[0] for f in N.AttnParams._fields_]
    prog = ['#include <stdio.h>', '#include <stddef.h>', '#include "chia_attn.h"',
            'int main(void){', 'printf("%zu\\n", sizeof(chia_attn_params_t));']
    prog += [f'printf("%zu\\n", offsetof(chia_attn_params_t, {f}));' for f in fields]
    prog += ['return 0;}']
    c = tmp_path / "layout.c"
    c.write_text("\n".join(prog))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(c), "-o", str(exe)],
                   check=True)
    vals = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True,
                                           check=True).stdout.split()]
    assert vals[0] == ctypes.sizeof(N.AttnParams)
    for f, off in zip(fields, vals[1:]):
        assert getattr(N.AttnParams, f).offset == off, f


def _valid_params():
    p = N.AttnParams()
    p.abi_version = N.ABI_VERSION
    p.dtype = N.DTYPE_BF16
    p.head_dim = 128
    p.norm = N.NORM_SOFTMAX
    p.mod = N.MOD_NONE
    p.batch, p.heads, p.seqlen_q, p.seqlen_kv = 2, 4, 256, 256
    for f in ("q", "k", "v", "o"):
        setattr(p, f, 0x10000)  # never dereferenced: validation fails first in each case
    for f in ("q_stride", "k_stride", "v_stride", "o_stride"):
        getattr(p, f)[:] = (4 * 256 * 128, 256 * 128, 128)
    p.scale = 0.088
    p.softcap = 30.0
    p.out_scale = 1.0
    p.win_left, p.win_right, p.dilation = -1, 0, 1
    return p


@pytest.mark.parametrize("mutate,code", [
    (lambda p: setattr(p, "abi_version", 0), 1),
    (lambda p: setattr(p, "head_dim", 96), 2),
    (lambda p: setattr(p, "dtype", 7), 2),
    (lambda p: setattr(p, "norm", 9), 1),
    (lambda p: setattr(p, "mod", 9), 1),
    (lambda p: (setattr(p, "norm", N.NORM_RELU), setattr(p, "mod", N.MOD_SOFTCAP)), 2),
    (lambda p: setattr(p, "seqlen_q", 0), 1),
    (lambda p: setattr(p, "batch", -1), 1),
    (lambda p: setattr(p, "q", None), 1),
    (lambda p: setattr(p, "o", 0x10008), 3),
    (lambda p: p.k_stride.__setitem__(2, 100), 3),
    (lambda p: setattr(p, "dilation", 0), 1),
    (lambda p: setattr(p, "win_left", -2), 1),
    (lambda p: setattr(p, "mod", N.MOD_ALIBI), 1),   # ALiBi without slopes
    (lambda p: (setattr(p, "mod", N.MOD_SOFTCAP), setattr(p, "softcap", 0.0)), 1),
    (lambda p: setattr(p, "scale", float("nan")), 1),
    (lambda p: setattr(p, "heads_kv", 3), 1),    # 4 query heads, 3 K/V heads
    (lambda p: setattr(p, "heads_kv", -1), 1),
    (lambda p: setattr(p, "lse", 0x30002), 3),   # log-sum-exp output not 4-byte aligned
    # packed sequences: batch must be 1 ...
    (lambda p: (setattr(p, "seq_offsets", 0x20000), setattr(p, "num_seqs", 2)), 1),
    # ... a prefix (or block, dilation) is not supported with them ...
    (lambda p: (setattr(p, "batch", 1), setattr(p, "seq_offsets", 0x20000),
                setattr(p, "num_seqs", 2), setattr(p, "prefix", 8)), 2),
    # ... the offsets are int32 ...
    (lambda p: (setattr(p, "batch", 1), setattr(p, "seq_offsets", 0x20002),
                setattr(p, "num_seqs", 2)), 3),
    (lambda p: (setattr(p, "batch", 1), setattr(p, "seq_offsets", 0x20000),
                setattr(p, "num_seqs", 0)), 1),
])
def test_argument_errors_are_reported_before_launch(lib, mutate, code):
    p = _valid_params()
    mutate(p)
    assert lib.chia_attn_fwd(ctypes.byref(p), None) == code
    assert lib.chia_attn_fwd(None, None) == 1


def test_host_helpers_reject_bad_masks(lib):
    p = _valid_params()
    p.dilation = 0
    assert lib.chia_attn_visible_pairs(ctypes.byref(p)) == -1
    lo, hi, bits = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_uint64()
    assert lib.chia_attn_tile_plan(ctypes.byref(p), 0, 128, 128, ctypes.byref(lo),
                                   ctypes.byref(hi), ctypes.byref(bits)) == 1
    # packed-sequence offsets live in device memory: the host helpers decline
    p = _valid_params()
    p.batch, p.seq_offsets, p.num_seqs = 1, 0x20000, 2
    assert lib.chia_attn_visible_pairs(ctypes.byref(p)) == -1
    assert lib.chia_attn_tile_plan(ctypes.byref(p), 0, 128, 128, ctypes.byref(lo),
                                   ctypes.byref(hi), ctypes.byref(bits)) == 2


def test_python_api_has_no_cpu_fallback(lib):
    import torch
    import chia_proj_b200 as cp
    q = torch.randn(1, 1, 16, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        cp.softcap_gemma2(q, q, q)
    with pytest.raises(ValueError):
        cp.bias_sliding_window(q, q, q, window=0)
