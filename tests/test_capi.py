"""C ABI checks that need no GPU: exports, registry metadata, argument guards.

Every guard in swiglu_b200.h runs before any CUDA call, so invalid calls are
exercised here with fake pointers; nothing is launched.
"""
import ctypes
import subprocess

import pytest

from swiglu_b200 import _lib

FAKE = 0x7F0000000000  # never dereferenced: every call below fails a guard first


def L():
    return _lib.lib()


def test_library_exports_every_declared_symbol():
    declared = _lib.declared_symbols()
    api_lines = sum(h.read_text().count("\nSWB_API ") for h in _lib.HEADERS)
    assert len(declared) == api_lines >= 19
    for path in (_lib.LIB_PATH, _lib.CUBLAS_LIB_PATH):
        out = subprocess.run(["nm", "-D", "--defined-only", str(path)], capture_output=True, text=True, check=True)
        exported = {line.split()[-1] for line in out.stdout.splitlines() if " T " in line}
        mine = [s for s in declared if (s.startswith("swbl_") == (path == _lib.CUBLAS_LIB_PATH))]
        missing = [s for s in mine if s not in exported]
        assert not missing, (path.name, missing)
        # nothing but the declared C ABI leaks out of the product library
        assert exported <= set(declared), exported - set(declared)
    for s in declared:
        assert hasattr(_lib.cublas_lib() if s.startswith("swbl_") else L(), s)


def test_library_is_sm100a_only_and_self_contained():
    out = subprocess.run(["ldd", str(_lib.LIB_PATH)], capture_output=True, text=True, check=True).stdout
    assert "libcudart" not in out  # runtime linked statically: nothing to resolve on the box
    assert "libcublas" not in out  # the product path does not depend on cuBLAS


def test_status_strings_match_reference_messages():
    expected = {
        1: "invalid projection input", 2: "invalid gate buffers", 3: "missing half output",
        4: "missing float output", 5: "missing residual", 6: "unknown kernel configuration",
        7: "invalid shape", 8: "configuration out of range", 9: "invalid configuration",
        10: "workspace overlaps input storage", 11: "scratch and output overlap",
    }
    for code, msg in expected.items():
        assert _lib.status_message(code) == msg


def test_registry_keeps_reference_ids_and_rejects_invalid():
    from swiglu_b200 import config_ids, valid_config, config_info
    ids = config_ids()
    assert ids[:10] == [1, 2, 4, 8, 16, 17, 18, 19, 20, 21]  # include/config.hpp:7-9
    assert len(ids) == len(set(ids)) == L().swb_config_count()
    for bad in (0, 999, 1000, -1, 2 ** 32 + 1):
        assert not valid_config(bad)
    ref_geom = {1: (1, 4, 2), 2: (2, 4, 2), 4: (4, 4, 2), 8: (8, 4, 2), 16: (1, 4, 8), 17: (2, 4, 8),
                18: (4, 2, 8), 19: (1, 8, 8), 20: (2, 2, 8), 21: (4, 1, 8)}
    for cid in ids:
        c = config_info(cid)
        assert c["id"] == cid
        if c["family"] == _lib.SWB_FAMILY_LDG:
            assert c["warps"] * c["rows"] * 32 <= 1024 and c["pack"] in (2, 8)
            assert c["chunk"] == 0 and c["stages"] == 0
        elif c["family"] == _lib.SWB_FAMILY_BULK:
            assert c["chunk"] % 8 == 0 and c["stages"] >= 2 and (c["warps"] + 1) * 32 <= 1024
        else:
            assert c["family"] in (_lib.SWB_FAMILY_RBULK, _lib.SWB_FAMILY_SBULK)
            assert 1 <= c["unroll"] <= 8 and c["stages"] >= 2 and (c["warps"] + 1) * 32 <= 1024
        if cid in ref_geom:
            assert (c["warps"], c["rows"], c["pack"]) == ref_geom[cid]
    with pytest.raises(RuntimeError, match="unknown kernel configuration"):
        config_info(999)


def _msg():
    return _lib.last_error()


def test_gate_guards_in_reference_order():
    f = L().swb_gate
    assert f(1, None, FAKE, FAKE, None, None, FAKE, 4, 4, 0, None) == _lib.SWB_E_INPUT
    assert f(1, FAKE, FAKE, FAKE, None, None, FAKE, 0, 4, 0, None) == _lib.SWB_E_INPUT
    assert f(1, FAKE, FAKE, None, None, None, FAKE, 4, 4, 0, None) == _lib.SWB_E_INPUT
    assert f(1, FAKE, None, FAKE, None, None, FAKE, 4, 4, 0, None) == _lib.SWB_E_GATE_BUFFERS
    assert f(1, FAKE, FAKE, FAKE, None, None, None, 4, 4, 0, None) == _lib.SWB_E_GATE_BUFFERS
    assert f(999, FAKE, FAKE, FAKE, None, None, FAKE, 4, 4, 0, None) == _lib.SWB_E_CONFIG
    assert _msg() == "unknown kernel configuration"


def test_project_guards_in_reference_order():
    f = L().swb_project
    assert f(1, None, FAKE, None, None, FAKE, 4, 4, 0, None) == _lib.SWB_E_INPUT
    assert f(1, FAKE, FAKE, None, None, None, 4, 4, 0, None) == _lib.SWB_E_FLOAT_OUTPUT
    assert f(1, FAKE, FAKE, None, None, None, 4, 4, _lib.SWB_HALF_OUT, None) == _lib.SWB_E_HALF_OUTPUT
    assert f(1, FAKE, FAKE, None, None, FAKE, 4, 4, _lib.SWB_RESIDUAL, None) == _lib.SWB_E_RESIDUAL
    assert f(0, FAKE, FAKE, None, None, FAKE, 4, 4, 0, None) == _lib.SWB_E_CONFIG


def test_swiglu_out_guards_in_binding_order():
    f = L().swb_swiglu_out
    H, I = 64, 96
    x, g, u, d, h, y = (FAKE + k * (1 << 24) for k in range(6))
    assert f(x, g, u, d, h, y, 0, I, 1, 1, None) == _lib.SWB_E_SHAPE
    assert f(x, g, u, d, h, y, H, 100001, 1, 1, None) == _lib.SWB_E_SHAPE
    # configuration ids are range-checked before narrowing (torch_extension.cu:21-22)
    assert f(x, g, u, d, h, y, H, I, 2 ** 32 + 1, 1, None) == _lib.SWB_E_CONFIG_RANGE
    assert f(x, g, u, d, h, y, H, I, 1, -1, None) == _lib.SWB_E_CONFIG_RANGE
    assert f(x, g, u, d, h, y, H, I, 0, 1, None) == _lib.SWB_E_CONFIG_INVALID
    assert f(x, g, u, d, h, y, H, I, 1, 999, None) == _lib.SWB_E_CONFIG_INVALID
    assert _msg() == "invalid configuration"
    # aliasing: output onto the input x, h onto a weight, h onto y
    assert f(x, g, u, d, h, x, H, I, 1, 1, None) == _lib.SWB_E_OVERLAP_INPUT
    assert f(x, g, u, d, g + 10, y, H, I, 1, 1, None) == _lib.SWB_E_OVERLAP_INPUT
    assert f(x, g, u, d, h, h + 2 * I - 2, H, I, 1, 1, None) == _lib.SWB_E_OVERLAP_OUTPUT
    assert _msg() == "scratch and output overlap"
    # adjacent but disjoint buffers are accepted by the alias guard (then fail null checks)
    assert f(x, g, u, d, h, None, H, I, 1, 1, None) == _lib.SWB_E_HALF_OUTPUT


def test_ffn_guards():
    f = L().swb_ffn
    assert f(1, 999, FAKE, FAKE, FAKE, FAKE, None, None, None, FAKE, FAKE, 8, 8, None) == _lib.SWB_E_CONFIG
    assert f(1, 1, FAKE, FAKE, None, FAKE, None, None, None, FAKE, FAKE, 8, 8, None) == _lib.SWB_E_INPUT
    assert f(1, 1, FAKE, FAKE, FAKE, FAKE, None, None, None, FAKE, None, 8, 8, None) == _lib.SWB_E_FLOAT_OUTPUT
    # launch flags: unknown bits are rejected first, before any CUDA call
    fx = L().swb_ffn_ex
    assert fx(1, 1, FAKE, FAKE, FAKE, FAKE, None, None, None, FAKE, FAKE, 8, 8, 2, None) == _lib.SWB_E_INPUT
    assert b"unknown launch flags" in L().swb_last_error()
    assert fx(1, 999, FAKE, FAKE, FAKE, FAKE, None, None, None, FAKE, FAKE, 8, 8,
              _lib.SWB_PREFETCH_WEIGHTS, None) == _lib.SWB_E_CONFIG


def test_epilogue_guards():
    assert L().swb_gate_epilogue(None, FAKE, FAKE, FAKE, FAKE, 8, None) == _lib.SWB_E_INPUT
    assert L().swb_residual_epilogue(FAKE, FAKE, FAKE, 0, None) == _lib.SWB_E_INPUT


def test_binding_rejects_cpu_tensors_with_reference_message():
    import torch
    from swiglu_b200 import swiglu_out, swiglu
    t = torch.zeros(4, dtype=torch.float16)
    w = torch.zeros(4, 4, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="all buffers must be contiguous CUDA FP16 tensors"):
        swiglu_out(t, w, w, w, t.clone(), t.clone(), 1, 1)
    with pytest.raises(RuntimeError, match="gate must be a matrix"):
        swiglu(t, t, w, w, 1)
    with pytest.raises(TypeError):
        swiglu_out(t, w, w, w, t, t, 2 ** 64, 1)


def test_decode_swiglu_dropin_module():
    import decode_swiglu as ext
    from swiglu_b200 import binding
    assert ext.swiglu_out is binding.swiglu_out and ext.swiglu is binding.swiglu
    assert ext.config_ids() == binding.config_ids()


def test_tp_exchange_guards_without_gpu():
    out = ctypes.c_void_p()
    for rank, world, rows in ((0, 0, 16), (0, 9, 16), (2, 2, 16), (-1, 2, 16), (0, 2, 0)):
        assert L().swb_tp_create(rank, world, rows, ctypes.byref(out)) == _lib.SWB_E_INPUT
    assert L().swb_tp_ipc_handle(None, None) == _lib.SWB_E_INPUT
    assert L().swb_tp_connect(None, None) == _lib.SWB_E_INPUT
    assert L().swb_tp_destroy(None) == _lib.SWB_OK
    f = L().swb_ffn_tp_fused
    assert f(None, 83, 83, *([FAKE] * 9), 64, 32, None) == _lib.SWB_E_INPUT
    fx = L().swb_ffn_tp_fused_ex
    assert fx(None, 83, 83, *([FAKE] * 9), 64, 32, 4, None) == _lib.SWB_E_INPUT
    assert b"unknown launch flags" in L().swb_last_error()
    assert fx(None, 83, 83, *([FAKE] * 9), 64, 32, _lib.SWB_PREFETCH_WEIGHTS, None) == _lib.SWB_E_INPUT


def test_ctypes_declarations_match_header_arity():
    """Every typed entry point takes exactly as many arguments as the header declares."""
    sigs = _lib.declared_signatures()
    assert len(sigs) == len(_lib.declared_symbols())
    for name, nparams in sigs.items():
        fn = getattr(_lib.cublas_lib() if name.startswith("swbl_") else L(), name)
        assert fn.argtypes is not None, name
        assert len(fn.argtypes) == nparams, (name, len(fn.argtypes), nparams)


def test_layer_registry_and_fused_guards():
    from swiglu_b200 import layer_config_ids
    ids = layer_config_ids()
    assert ids[:2] == [200, 203] and all(i >= 200 for i in ids)
    assert not set(ids) & set(__import__("swiglu_b200").config_ids())
    f = L().swb_ffn_fused
    assert f(33, *([FAKE] * 9), 64, 96, FAKE, None) == _lib.SWB_E_CONFIG        # projection id, not a layer id
    assert f(200, *([FAKE] * 9), 64, 96, None, None) == _lib.SWB_E_WORKSPACE
    assert f(200, *([FAKE] * 9), 64, 96, ctypes.c_void_p(0x1004), None) == _lib.SWB_E_WORKSPACE  # misaligned
    assert b"16-byte aligned" in L().swb_last_error()
    assert f(200, None, *([FAKE] * 8), 64, 96, FAKE, None) == _lib.SWB_E_INPUT
    assert f(200, FAKE, None, *([FAKE] * 7), 64, 96, FAKE, None) == _lib.SWB_E_GATE_BUFFERS
    # the streaming ids are layer ids too; the flags variant rejects unknown bits first
    assert {220, 221, 223} <= set(ids)
    fx = L().swb_ffn_fused_ex
    assert fx(220, *([FAKE] * 9), 64, 96, FAKE, 2, None) == _lib.SWB_E_INPUT
    assert b"flags" in L().swb_last_error()
    assert fx(33, *([FAKE] * 9), 64, 96, FAKE, _lib.SWB_PREFETCH_WEIGHTS, None) == _lib.SWB_E_CONFIG
    assert fx(220, *([FAKE] * 9), 64, 96, None, _lib.SWB_PREFETCH_WEIGHTS, None) == _lib.SWB_E_WORKSPACE


def test_tp_model_path_and_epoch_guards_without_gpu():
    """swb_swiglu_tp_out and swb_tp_epoch refuse a missing exchange, and unknown flags, before
    any CUDA call."""
    f = L().swb_swiglu_tp_out
    assert f(None, *([FAKE] * 6), 4096, 512, 69, 87, 0, None) == _lib.SWB_E_INPUT
    assert b"exchange" in L().swb_last_error()
    assert f(FAKE, *([FAKE] * 6), 4096, 512, 69, 87, 4, None) == _lib.SWB_E_INPUT  # unknown flag bit
    assert b"flags" in L().swb_last_error()
    out = ctypes.c_uint32()
    assert L().swb_tp_epoch(None, ctypes.byref(out)) == _lib.SWB_E_INPUT
    assert L().swb_tp_epoch(FAKE, None) == _lib.SWB_E_INPUT
    fh = L().swb_ffn_tp_host_ex
    assert fh(None, 69, 102, *([FAKE] * 11), 4096, 512, 0, None) == _lib.SWB_E_INPUT
    assert b"exchange" in L().swb_last_error()
    assert fh(None, 69, 102, *([FAKE] * 11), 4096, 512, 8, None) == _lib.SWB_E_INPUT  # unknown flag bit
    assert b"flags" in L().swb_last_error()


def test_host_buffer_layer_guards_without_gpu():
    """swb_ffn_host_ex refuses unknown flags, invalid geometries, missing or aliased buffers and
    host pointers that are not page-locked host memory -- all before any launch."""
    f = L().swb_ffn_host_ex
    x, h, y = 0x7F0000100000, 0x7F0000200000, 0x7F0000300000

    def call(g=69, d=101, wg=FAKE, wu=FAKE, wd=FAKE, xh=FAKE, xd=x, hd=h, yd=y, yh=FAKE, hidden=64, inter=96,
             flags=0):
        return f(g, d, wg, wu, wd, xh, None, None, None, xd, hd, yd, yh, hidden, inter, flags, None)

    assert call(flags=2) == _lib.SWB_E_INPUT
    assert b"flags" in L().swb_last_error()
    assert call(g=999) == _lib.SWB_E_CONFIG
    assert call(d=0) == _lib.SWB_E_CONFIG
    assert call(xh=None) == _lib.SWB_E_INPUT
    assert call(xd=None) == _lib.SWB_E_INPUT
    assert call(hidden=0) == _lib.SWB_E_INPUT
    assert call(wu=None) == _lib.SWB_E_GATE_BUFFERS
    assert call(hd=None) == _lib.SWB_E_GATE_BUFFERS
    assert call(yd=None) == _lib.SWB_E_FLOAT_OUTPUT
    assert call(yh=None) == _lib.SWB_E_FLOAT_OUTPUT
    assert call(hd=x + 64) == _lib.SWB_E_OVERLAP_OUTPUT          # h inside x's 128 bytes
    assert call(yd=h + 100) == _lib.SWB_E_OVERLAP_OUTPUT         # y inside h's 192 bytes
    # not page-locked host memory (here: not memory at all): refused on the host
    assert call() == _lib.SWB_E_INPUT
    assert b"page-locked" in L().swb_last_error()
    assert call(flags=_lib.SWB_PREFETCH_WEIGHTS) == _lib.SWB_E_INPUT


C_CALLER = r"""
#include <stdio.h>
#include <string.h>
#include "swiglu_b200.h"

#define EXPECT(cond) do { if (!(cond)) { printf("FAIL line %d\n", __LINE__); return 1; } } while (0)

int main(void) {
    /* the registry, as decode_bench would iterate it */
    int n = swb_config_count();
    EXPECT(n > 10);
    int ids[256];
    EXPECT(swb_config_ids(ids, 256) == n);
    EXPECT(ids[0] == 1 && swb_valid_config(1) && !swb_valid_config(0) && !swb_valid_config(999));
    swb_config_t c;
    EXPECT(swb_config_info(17, &c) == SWB_OK && c.id == 17 && c.warps == 2 && c.rows == 4 && c.pack == 8);
    /* guards run before any CUDA call: no GPU is needed for these */
    void* fake = (void*)0x7f0000000000ull;
    float* yf = (float*)fake;
    EXPECT(swb_ffn(1, 999, fake, fake, fake, fake, NULL, NULL, NULL, fake, yf, 8, 8, NULL) == SWB_E_CONFIG);
    EXPECT(strcmp(swb_status_string(SWB_E_CONFIG), "unknown kernel configuration") == 0);
    EXPECT(swb_ffn_ex(1, 1, fake, fake, fake, fake, NULL, NULL, NULL, fake, yf, 8, 8, 2u, NULL) == SWB_E_INPUT);
    EXPECT(strstr(swb_last_error(), "unknown launch flags") != NULL);
    EXPECT(swb_swiglu_out(fake, fake, fake, fake, fake, fake, 8, 8, 1001, 1, NULL) == SWB_E_CONFIG_RANGE);
    swb_tp_t* tp = NULL;
    EXPECT(swb_tp_create(0, 9, 16, &tp) == SWB_E_INPUT && tp == NULL);
    EXPECT(swb_tp_destroy(NULL) == SWB_OK);
    puts("C caller ok");
    return 0;
}
"""


def test_header_is_plain_c_and_the_library_links(tmp_path):
    """A C11 caller with no Python and no C++ compiles against the header, links the library
    and gets the registry and the guards' codes and messages."""
    import shutil
    import subprocess
    if not shutil.which("gcc"):
        pytest.skip("gcc not available")
    src = tmp_path / "caller.c"
    src.write_text(C_CALLER)
    exe = tmp_path / "caller"
    libdir = _lib.LIB_PATH.parent
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", f"-I{_lib.REPO_ROOT / 'include'}", str(src),
                    f"-L{libdir}", "-lswiglu_b200", f"-Wl,-rpath,{libdir}", "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0 and "C caller ok" in out.stdout, out.stdout + out.stderr
