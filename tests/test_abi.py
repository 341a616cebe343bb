"""The C ABI of libqmla.so without a GPU: it loads, exports every function include/qmla.h
declares, its parameter struct has the header's layout, and the host-only entry points
(qmla_plan, qmla_error_string, qmla_abi_version) are exact."""
from __future__ import annotations

import ctypes
import pathlib
import re
import shutil
import subprocess

import numpy as np
import pytest

import oracle
from conftest import ROOT
from qwen_mla_vllm_b200 import _lib

HEADER = ROOT / "include" / "qmla.h"


def _declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(qmla_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    return _lib.load()


def test_exports_every_declared_symbol(lib):
    names = _declared_functions()
    assert len(names) >= 9, names
    for n in names:
        assert hasattr(lib, n), f"{n} declared in qmla.h but not exported"
    assert set(names) <= set(_lib.PROTOTYPES), set(names) - set(_lib.PROTOTYPES)


def test_abi_version_and_errors(lib):
    assert lib.qmla_abi_version() == 103
    for code, text in _lib.ERRORS.items():
        assert lib.qmla_error_string(code).decode() == text
    assert lib.qmla_error_string(0).decode() == "ok"


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
@pytest.mark.parametrize("cname,pystruct", [("qmla_decode_params", _lib.DecodeParams),
                                            ("qmla_dcp_p2p_params", _lib.DcpP2PParams),
                                            ("qmla_gather_params", _lib.GatherParams)])
def test_params_struct_layout_matches_header(tmp_path, cname, pystruct):
    fields = [f for f, _ in pystruct._fields_]
    src = ["#include <stdio.h>", "#include <stddef.h>", '#include "qmla.h"', "int main(void) {",
           f'printf("%zu\\n", sizeof({cname}));']
    src += [f'printf("%zu\\n", offsetof({cname}, {f}));' for f in fields]
    src += ["return 0; }"]
    c = tmp_path / "layout.c"
    c.write_text("\n".join(src))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", str(HEADER.parent), str(c), "-o", str(exe)], check=True)
    vals = [int(x) for x in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()]
    assert vals[0] == ctypes.sizeof(pystruct)
    for f, off in zip(fields, vals[1:]):
        assert getattr(pystruct, f).offset == off, f


def test_dcp_buffer_layout(lib):
    vals = [ctypes.c_int64() for _ in range(5)]
    assert lib.qmla_dcp_buffer_layout(64, 24, 768, *[ctypes.byref(v) for v in vals]) == 0
    total, o_off, o_slot, lse_off, lse_slot = (v.value for v in vals)
    assert o_off == 256 and o_slot == 64 * 24 * 768 * 4
    assert lse_off == o_off + 2 * o_slot and lse_slot == 6144
    assert total == lse_off + 2 * lse_slot
    assert lib.qmla_dcp_buffer_layout(-1, 24, 768, *[ctypes.byref(v) for v in vals]) == -1


def test_gather_rejects_bad_arguments_without_launching(lib):
    """Argument checks run on the host before any launch (no GPU needed)."""
    p = _lib.GatherParams()
    assert lib.qmla_gather_cache(None, None) == -1
    p.num_tokens = 0
    assert lib.qmla_gather_cache(ctypes.byref(p), None) == 0          # nothing to gather
    p.num_tokens = -1
    assert lib.qmla_gather_cache(ctypes.byref(p), None) == -1
    p.num_tokens, p.num_seqs = 4, 1
    assert lib.qmla_gather_cache(ctypes.byref(p), None) == -1         # null pointers
    fake = 1 << 20  # never dereferenced: every call below fails its host checks first
    p.src_cache = p.dst = p.block_table = p.cu_seq_lens = p.token_to_seq = fake
    p.page_size, p.num_pages, p.block_table_cols = 16, 8, 4
    p.src_dtype, p.dst_dtype = _lib.DT_F32, _lib.DT_BF16
    assert lib.qmla_gather_cache(ctypes.byref(p), None) == -2         # f32 cache
    p.src_dtype, p.dst_dtype = _lib.DT_FP8E4M3, _lib.DT_FP8E4M3
    assert lib.qmla_gather_cache(ctypes.byref(p), None) == -2         # FP8 destination
    p.dst_dtype = _lib.DT_BF16
    p.rms_offset, p.rms_heads, p.rms_mode = 1000, 24, _lib.RMS_LOG8
    assert lib.qmla_gather_cache(ctypes.byref(p), None) == -1         # FP8 without a scale
    p.scale = fake
    p.src_stride_token, p.src_stride_page, p.dst_stride_row = 1020, 16 * 1020, 1024
    assert lib.qmla_gather_cache(ctypes.byref(p), None) == -1         # row shorter than off + heads
    p.src_stride_token, p.src_stride_page, p.dst_stride_row = 1024, 16 * 1024, 1000
    assert lib.qmla_gather_cache(ctypes.byref(p), None) == -1         # destination too narrow
    p.dst_stride_row, p.rms_mode = 1024, 7
    assert lib.qmla_gather_cache(ctypes.byref(p), None) == -1         # unknown rms mode


def _plan(lib, lens, page):
    n = len(lens)
    sl = np.ascontiguousarray(lens, dtype=np.int32)
    tp = np.zeros(n + 1, np.int32)
    ip = np.zeros(n + 1, np.int32)
    kl = np.zeros(max(n, 1), np.int32)
    tt, tpg = ctypes.c_int64(), ctypes.c_int64()
    rc = lib.qmla_plan(sl.ctypes.data, n, page, tp.ctypes.data, ip.ctypes.data, kl.ctypes.data,
                       ctypes.byref(tt), ctypes.byref(tpg))
    return rc, tp, ip, kl[:n], tt.value, tpg.value


@pytest.mark.parametrize("page", [1, 16, 64, 400, 784])
def test_qmla_plan_exact(lib, page):
    rng = np.random.default_rng(page)
    lens = np.concatenate([[0, -3, 1, 63, 64, 65], rng.integers(1, 70000, 200)]).astype(np.int32)
    rc, tp, ip, kl, tt, tpg = _plan(lib, lens, page)
    assert rc == 0
    otp, oip, okl = oracle.plan_arrays(lens, page)
    assert np.array_equal(tp, otp) and np.array_equal(ip, oip) and np.array_equal(kl, okl)
    assert tt == otp[-1] and tpg == oip[-1]


def test_qmla_plan_rejects_bad_args(lib):
    lens = np.array([5], np.int32)
    tp = np.zeros(2, np.int32)
    assert lib.qmla_plan(None, 1, 16, tp.ctypes.data, None, None, None, None) == _lib_code("INVALID")
    assert lib.qmla_plan(lens.ctypes.data, 1, 0, tp.ctypes.data, None, None, None, None) == _lib_code("INVALID")
    assert lib.qmla_plan(lens.ctypes.data, 0, 16, tp.ctypes.data, None, None, None, None) == 0
    # overflow of the int32 page prefix is reported, not wrapped
    big = np.full(3, 2**31 - 1, np.int32)
    tp3 = np.zeros(4, np.int32)
    ip3 = np.zeros(4, np.int32)
    assert lib.qmla_plan(big.ctypes.data, 3, 1, tp3.ctypes.data, ip3.ctypes.data, None, None, None) == _lib_code("UNSUPPORTED")


def _lib_code(name):
    return {"INVALID": -1, "UNSUPPORTED": -2, "ALIGNMENT": -3, "WORKSPACE": -4, "CUDA": -5}[name]


def test_launching_entry_points_validate_before_touching_cuda(lib):
    # null parameter blocks and bad sizes are rejected on the host
    assert lib.qmla_mla_decode(None, None) == -1
    n = ctypes.c_int64()
    assert lib.qmla_decode_workspace_bytes(None, ctypes.byref(n)) == -1
    assert lib.qmla_dcp_merge(None, 2, None, None, 0, None, 2, 1, 1, 1, None) == -1
    assert lib.qmla_dcp_correct(None, 2, 0, 0, None, 0, 0, None, 2, 0, 1, 1, 1, 1, None) == -1
    assert lib.qmla_fp8_cache_write(None, 0, None, 0, None, 1, 1, 1, 1, 3, None, None, 1, None) == -1


def test_status_bits_match_binding():
    """QMLA_STATUS_* in qmla.h are the bits the Python binding tests for."""
    bits = dict(re.findall(r"#define QMLA_STATUS_(\w+) (\d+)", HEADER.read_text()))
    assert int(bits["TIMEOUT"]) == _lib.DEV_ERR_TIMEOUT
    assert int(bits["BAD_INDEX"]) == _lib.DEV_ERR_INDEX
