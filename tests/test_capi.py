"""The C ABI without a GPU: libsas.so loads, exports every function that
include/sas.h declares, and the ctypes mirror in ``_lib`` agrees with the
header on struct layouts and constants (checked against a small C program
compiled from the header with gcc).  Host-only entry points (scheduler,
planner, workspace sizing, error strings) are called; nothing launches."""

import ctypes as C
import os
import re
import shutil
import subprocess

import pytest

from sparse_attn_sharedkv_b200 import _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "sas.h")


def _declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(sas_[a-z_0-9]+)\s*\(", text,
                       flags=re.M)
    return sorted(set(names))


def test_header_declares_the_expected_entry_points():
    names = _declared_functions()
    for n in ("sas_fwd", "sas_fwd_prepare", "sas_fwd_execute", "sas_fwd_workspace_size",
              "sas_fwd_noalloc", "sas_combine", "sas_metadata", "sas_plan", "sas_plan_size",
              "sas_error_string", "sas_version", "sas_device_sm_count"):
        assert n in names


def test_library_exports_every_declared_function():
    L = _lib.lib()
    missing = [n for n in _declared_functions() if not hasattr(L, n)]
    assert not missing, missing
    # and the ctypes prototypes cover the same set
    assert set(_lib.PROTOTYPES) == set(_declared_functions())


def test_nm_shows_c_linkage():
    if shutil.which("nm") is None:
        pytest.skip("nm not available")
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    for n in _declared_functions():
        assert n in exported, n          # unmangled: extern "C"


_PROBE = r"""
#include <stdio.h>
#include <stddef.h>
#include "sas.h"
#define S(T) printf(#T " size %zu\n", sizeof(T));
#define F(T, f) printf(#T " " #f " %zu\n", offsetof(T, f));
#define K(c) printf("const " #c " %lld\n", (long long)(c));
int main(void) {
  S(SasMetaParams) S(SasProblem) S(SasFwdParams) S(SasPlanInfo)
  F(SasMetaParams, cu_seqlens_q) F(SasMetaParams, ori_mask_mode) F(SasMetaParams, ori_win_left)
  F(SasMetaParams, layout_q) F(SasMetaParams, has_ori_kv) F(SasMetaParams, aiv_core_num)
  F(SasProblem, q_start) F(SasProblem, num_heads) F(SasProblem, topk)
  F(SasFwdParams, err) F(SasFwdParams, head_dim) F(SasFwdParams, softmax_scale)
  F(SasFwdParams, cmp_table_len) F(SasFwdParams, num_sms) F(SasFwdParams, trace)
  F(SasFwdParams, slot_dump) F(SasFwdParams, slot_dump_cap)
  F(SasPlanInfo, total_tiles) F(SasPlanInfo, actkv_off)
  K(SAS_OK) K(SAS_ERR_INVALID) K(SAS_ERR_UNSUPPORTED) K(SAS_ERR_CUDA) K(SAS_ERR_SCHEDULE)
  K(SAS_ERR_WORKSPACE) K(SAS_ERR_DEVICE) K(SAS_DTYPE_BF16) K(SAS_DTYPE_FP16)
  K(SAS_LAYOUT_BSND) K(SAS_LAYOUT_TND) K(SAS_SCENARIO_SWA) K(SAS_SCENARIO_CFA)
  K(SAS_SCENARIO_SCFA) K(SAS_PHASE_ATTN) K(SAS_PHASE_COMBINE) K(SAS_PHASE_ALL)
  K(SAS_META_SIZE) K(SAS_NOALLOC_SCRATCH_BYTES)
  return 0;
}
"""


@pytest.fixture(scope="module")
def header_probe(tmp_path_factory):
    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    d = tmp_path_factory.mktemp("abi")
    src, exe = d / "probe.c", d / "probe"
    src.write_text(_PROBE)
    subprocess.run(["gcc", "-std=c99", "-I", os.path.join(REPO, "include"), str(src), "-o",
                    str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    sizes, offsets, consts = {}, {}, {}
    for line in out.splitlines():
        a, b, c = line.split()
        if b == "size":
            sizes[a] = int(c)
        elif a == "const":
            consts[b] = int(c)
        else:
            offsets[(a, b)] = int(c)
    return sizes, offsets, consts


def test_ctypes_structs_match_header(header_probe):
    sizes, offsets, _ = header_probe
    for name, size in sizes.items():
        assert C.sizeof(getattr(_lib, name)) == size, name
    for (struct, field), off in offsets.items():
        assert getattr(getattr(_lib, struct), field).offset == off, (struct, field)


def test_ctypes_constants_match_header(header_probe):
    _, _, k = header_probe
    assert k["SAS_OK"] == _lib.SAS_OK
    for code, name in _lib.ERRORS.items():
        assert k[name] == code
    assert (k["SAS_DTYPE_BF16"], k["SAS_DTYPE_FP16"]) == (_lib.DTYPE_BF16, _lib.DTYPE_FP16)
    assert k["SAS_LAYOUT_BSND"] == _lib.LAYOUTS["BSND"]
    assert k["SAS_LAYOUT_TND"] == _lib.LAYOUTS["TND"]
    assert (k["SAS_SCENARIO_SWA"], k["SAS_SCENARIO_CFA"], k["SAS_SCENARIO_SCFA"]) == (
        _lib.SCENARIO_SWA, _lib.SCENARIO_CFA, _lib.SCENARIO_SCFA)
    assert (k["SAS_PHASE_ATTN"], k["SAS_PHASE_COMBINE"], k["SAS_PHASE_ALL"]) == (
        _lib.PHASE_ATTN, _lib.PHASE_COMBINE, _lib.PHASE_ALL)
    assert k["SAS_META_SIZE"] == _lib.SAS_META_SIZE
    assert k["SAS_NOALLOC_SCRATCH_BYTES"] == _lib.SAS_NOALLOC_SCRATCH_BYTES


def test_error_strings_and_version():
    L = _lib.lib()
    for code in [0, *_lib.ERRORS]:
        s = L.sas_error_string(code)
        assert s and len(s) >= 2
    assert L.sas_version().decode().count(".") >= 1


def _problem(B=2, H=64, K=512, q_lens=(3, 2), kv_lens=(900, 700)):
    q_len = (C.c_int32 * B)(*q_lens)
    kv_len = (C.c_int32 * B)(*kv_lens)
    starts = [0]
    for x in q_lens[:-1]:
        starts.append(starts[-1] + x)
    q_start = (C.c_int32 * B)(*starts)
    prob = _lib.SasProblem(batch=B, layout_q=_lib.LAYOUTS["TND"], max_q_len=max(q_lens),
                           total_tokens=sum(q_lens), q_start=q_start, q_len=q_len,
                           kv_len=kv_len, num_heads=H, scenario=_lib.SCENARIO_SCFA,
                           ori_win_left=127, cmp_ratio=4, topk=K)
    return prob, (q_len, kv_len, q_start)


def test_workspace_size_and_plan_are_host_only():
    L = _lib.lib()
    prob, keep = _problem()
    n = C.c_size_t()
    assert L.sas_fwd_workspace_size(C.byref(prob), 16, C.byref(n)) == 0
    assert n.value > 0 and n.value % 256 == 0
    info = _lib.SasPlanInfo()
    assert L.sas_plan_size(C.byref(prob), 16, C.byref(info)) == 0
    assert info.num_workers == 16 and info.head_groups == 1 and info.num_rows == 5


def test_invalid_problems_are_rejected_on_the_host():
    L = _lib.lib()
    n = C.c_size_t()
    prob, keep = _problem(H=129)
    assert L.sas_fwd_workspace_size(C.byref(prob), 16, C.byref(n)) == 1
    prob, keep = _problem()
    prob.scenario = 7
    assert L.sas_fwd_workspace_size(C.byref(prob), 16, C.byref(n)) == 1
    assert L.sas_fwd_workspace_size(None, 16, C.byref(n)) == 1
    # the no-allocation forward validates before it touches any device state
    assert L.sas_fwd_noalloc(None, None, None) == 1
