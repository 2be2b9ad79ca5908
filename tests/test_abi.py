"""CPU checks of the C ABI: the library loads, exports every function include/am_q4.h
declares, its struct layouts match the header, and host-side validation rejects bad
arguments before any CUDA call."""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from conftest import ROOT, pkg

HEADER = ROOT / "include" / "am_q4.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|const char\*)\s+(am_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    lib = pkg._lib.load()
    names = declared_functions()
    assert len(names) >= 9
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(pkg._lib.EXPORTED_SYMBOLS)
    assert lib.am_abi_version() == pkg._lib.ABI_VERSION


def test_struct_layout_matches_header(tmp_path):
    src = tmp_path / "layout.c"
    src.write_text(r'''
#include <stdio.h>
#include <stddef.h>
#include "am_q4.h"
int main(void) {
  printf("%zu %zu %zu %zu %zu\n", sizeof(am_q4_cache), offsetof(am_q4_cache, capacity),
         offsetof(am_q4_cache, block_table), sizeof(am_attn_args), offsetof(am_attn_args, status));
  printf("%zu %zu %zu\n", offsetof(am_attn_args, scale), offsetof(am_attn_args, mask_stride_b),
         offsetof(am_attn_args, max_kv_len));
  return 0;
}
''')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()
    C, A = pkg._lib.Q4CacheDesc, pkg._lib.AttnArgs
    want = [ctypes.sizeof(C), C.capacity.offset, C.block_table.offset, ctypes.sizeof(A),
            A.status.offset, A.scale.offset, A.mask_stride_b.offset, A.max_kv_len.offset]
    assert [int(x) for x in out] == want


def test_host_validation_rejects_bad_arguments():
    lib = pkg._lib.load()
    # dim not a multiple of 64: rejected before any device work
    rc = lib.am_q4_quantize(None, 0, 4, 96, None, None, None, None)
    assert rc == pkg._lib.AM_ERR_INVALID
    assert b"dim" in lib.am_last_error()
    rc = lib.am_q4_quantize(None, 7, 4, 64, None, None, None, None)
    assert rc == pkg._lib.AM_ERR_INVALID
    # NULL cache
    rc = lib.am_q4_decode(None, None, None, 0, None)
    assert rc == pkg._lib.AM_ERR_INVALID
    # cache with a bad layout
    d = pkg._lib.Q4CacheDesc()
    for f in ("k_codes", "k_scales", "k_biases", "v_codes", "v_scales", "v_biases"):
        setattr(d, f, 4096)
    d.scale_dtype, d.layout, d.n_kv_heads, d.k_dim, d.v_dim = 0, 9, 8, 128, 128
    d.capacity = 256
    a = pkg._lib.AttnArgs()
    rc = lib.am_q4_decode(ctypes.byref(d), ctypes.byref(a), None, 0, None)
    assert rc == pkg._lib.AM_ERR_INVALID and b"layout" in lib.am_last_error()
    d.layout = 0
    d.capacity = 100  # not a multiple of 16
    rc = lib.am_q4_decode(ctypes.byref(d), ctypes.byref(a), None, 0, None)
    assert rc == pkg._lib.AM_ERR_INVALID and b"capacity" in lib.am_last_error()
    # unsupported head dims are reported as such (no CPU fallback)
    d.capacity, d.k_dim, d.v_dim, d.batch = 256, 320, 320, 1
    a.q, a.out, a.kv_len, a.batch, a.n_q_heads, a.q_len = 4096, 4096, 4096, 1, 8, 1
    rc = lib.am_q4_decode(ctypes.byref(d), ctypes.byref(a), None, 0, None)
    assert rc == pkg._lib.AM_ERR_UNSUPPORTED


def test_workspace_size_is_zero_for_single_chunk():
    lib = pkg._lib.load()
    d = pkg._lib.Q4CacheDesc()
    d.n_kv_heads, d.k_dim, d.v_dim = 8, 128, 128
    a = pkg._lib.AttnArgs()
    a.batch, a.n_q_heads, a.q_len, a.max_kv_len = 1, 32, 1, 0
    assert lib.am_q4_attention_workspace_bytes(ctypes.byref(d), ctypes.byref(a)) == 0


def test_kernels_refuse_cpu_tensors():
    torch = pytest.importorskip("torch")
    with pytest.raises(ValueError, match="CUDA"):
        pkg.quantize(torch.zeros(2, 64, dtype=torch.float16))


def test_prefill_stage_rejects_a_reversed_key_range():
    """am_q4_prefill_stage checks its key range on the host before any device work."""
    lib = pkg._lib.load()
    d = pkg._lib.Q4CacheDesc()
    for f in ("k_codes", "k_scales", "k_biases", "v_codes", "v_scales", "v_biases"):
        setattr(d, f, 4096)
    d.scale_dtype, d.layout, d.n_kv_heads, d.k_dim, d.v_dim = 0, 0, 8, 128, 128
    d.capacity, d.batch = 256, 1
    a = pkg._lib.AttnArgs()
    a.q, a.out, a.kv_len, a.batch, a.n_q_heads, a.q_len, a.max_kv_len = 4096, 4096, 4096, 1, 32, 64, 256
    for lo, hi in ((10, 5), (-1, 5)):
        rc = lib.am_q4_prefill_stage(ctypes.byref(d), ctypes.byref(a), lo, hi, None, 0, None)
        assert rc == pkg._lib.AM_ERR_INVALID and b"key range" in lib.am_last_error()
