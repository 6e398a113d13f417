"""The C-ABI library without a GPU: it loads, exports every symbol
include/mm4.h declares, and validates descriptors on the host. No compute
call is made here."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from example_matmul_metal4_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


def _declared_symbols():
    text = (ROOT / "include" / "mm4.h").read_text()
    return sorted(set(re.findall(r"MM4_API\s+[\w\s\*]+?\b(mm4_\w+)\s*\(", text)))


def test_library_loads_without_gpu_runtime_dependencies():
    lib = _lib.lib()
    assert lib.mm4_version() >= 100
    deps = subprocess.run(["ldd", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    assert "libcuda.so" not in deps and "libcudart" not in deps


def test_every_declared_symbol_is_exported_and_bound():
    syms = _declared_symbols()
    assert len(syms) >= 25
    lib = _lib.lib()
    for s in syms:
        assert hasattr(lib, s), s
        assert s in _lib.SIGNATURES, f"{s} has no ctypes signature"
    nm = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (mm4_\w+)", nm))
    assert set(syms) <= exported
    assert exported <= set(syms), f"undeclared exports: {exported - set(syms)}"


def test_status_strings():
    lib = _lib.lib()
    for code, name in [(0, b"MM4_OK"), (1, b"MM4_ERR_INVALID"), (5, b"MM4_ERR_TIMEOUT"), (6, b"MM4_ERR_WORKSPACE")]:
        assert lib.mm4_status_string(code) == name


def _gemm(**kw):
    d = _lib.GemmDesc(*(kw.get(n, v) for n, v in [("M", 64), ("N", 64), ("K", 64), ("transpose_left", 0),
                                                   ("transpose_right", 0), ("bias", 1), ("split_k", 1),
                                                   ("block_m", 0), ("block_n", 0), ("block_k", 0),
                                                   ("cooperative_simdgroups", 4), ("preemptive_simdgroups", 1),
                                                   ("swap_mn", 0)]))
    h = ctypes.c_void_p()
    rc = _lib.lib().mm4_gemm_plan_create(ctypes.byref(h), ctypes.byref(d))
    return rc, h


def test_gemm_plan_validation_and_dispatch():
    lib = _lib.lib()
    assert _gemm(M=0)[0] == _lib.MM4_ERR_INVALID
    assert _gemm(K=-3)[0] == _lib.MM4_ERR_INVALID
    assert _gemm(transpose_left=2)[0] == _lib.MM4_ERR_INVALID
    assert b"positive" in lib.mm4_last_error() or b"0 or 1" in lib.mm4_last_error()
    rc, h = _gemm(M=512, N=512, K=65536, split_k=32)
    assert rc == 0
    assert b"splitk" in lib.mm4_gemm_plan_kernel_name(h)
    # 256x512 CTA-pair split-K tiles (2 of them): fp32 [512][512] workspace + one 64-bit counter
    # per 128-row half tile, rounded to 256 bytes
    assert b"BN=512" in lib.mm4_gemm_plan_kernel_name(h) and b"pair" in lib.mm4_gemm_plan_kernel_name(h)
    assert lib.mm4_gemm_workspace_size(h) == ((512 * 512 * 4 + 2 * 2 * 8 + 255) // 256) * 256
    lib.mm4_gemm_plan_destroy(h)
    rc, h = _gemm(M=33, N=40, K=31, transpose_right=1)
    assert rc == 0 and b"simt" in lib.mm4_gemm_plan_kernel_name(h)
    assert lib.mm4_gemm_workspace_size(h) == 0
    lib.mm4_gemm_plan_destroy(h)


def test_conv_and_attention_plan_validation():
    lib = _lib.lib()
    h = ctypes.c_void_p()
    d2 = _lib.Conv2dDesc(1, 5, 5, 4, 8, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, _lib.WEIGHTS_HWIO, 0)
    assert lib.mm4_conv2d_plan_create(ctypes.byref(h), ctypes.byref(d2)) == 0
    assert lib.mm4_conv_output_elements(h) == 5 * 5 * 8
    lib.mm4_conv_plan_destroy(h)
    bad = _lib.Conv2dDesc(1, 5, 5, 4, 8, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, _lib.WEIGHTS_DHWIO, 0)
    assert lib.mm4_conv2d_plan_create(ctypes.byref(h), ctypes.byref(bad)) == _lib.MM4_ERR_INVALID
    empty = _lib.Conv2dDesc(1, 2, 2, 4, 8, 3, 3, 1, 1, 1, 1, 0, 0, 0, 0, _lib.WEIGHTS_HWIO, 0)
    assert lib.mm4_conv2d_plan_create(ctypes.byref(h), ctypes.byref(empty)) == _lib.MM4_ERR_INVALID
    d3 = _lib.Conv3dDesc(8, 16, 64, 64, 128, 128, 3, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, _lib.WEIGHTS_ODHWI, 1)
    assert lib.mm4_conv3d_plan_create(ctypes.byref(h), ctypes.byref(d3)) == 0
    assert lib.mm4_conv_output_elements(h) == 8 * 16 * 64 * 64 * 128
    lib.mm4_conv_plan_destroy(h)
    a = _lib.AttentionDesc(4, 16, 16, 4096, 4096, 128, 0.0, _lib.MM4_ATTN_BHSD)
    assert lib.mm4_attention_plan_create(ctypes.byref(h), ctypes.byref(a)) == 0
    lib.mm4_attention_plan_destroy(h)
    a = _lib.AttentionDesc(1, 6, 4, 64, 64, 128, 0.0, _lib.MM4_ATTN_BHSD)
    assert lib.mm4_attention_plan_create(ctypes.byref(h), ctypes.byref(a)) == _lib.MM4_ERR_INVALID
    a = _lib.AttentionDesc(1, 4, 4, 64, 64, 96, 0.0, _lib.MM4_ATTN_BHSD)
    assert lib.mm4_attention_plan_create(ctypes.byref(h), ctypes.byref(a)) == _lib.MM4_ERR_UNSUPPORTED


def test_conv_tap_row_dispatch(monkeypatch):
    """Stride-1 convs on the CTA-pair path with dilation-1 filters 2 or 3 taps wide read all kw taps
    from one activation box (kernel name "taprow"); MM4_CONV_TAPREUSE=0 turns it off."""
    lib = _lib.lib()

    def name2d(*dims):
        h = ctypes.c_void_p()
        assert lib.mm4_conv2d_plan_create(ctypes.byref(h), ctypes.byref(_lib.Conv2dDesc(*dims))) == 0
        n = lib.mm4_conv_plan_kernel_name(h)
        lib.mm4_conv_plan_destroy(h)
        return n

    base = (32, 56, 56, 256, 256, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, _lib.WEIGHTS_OHWI, 1)
    assert b"taprow" in name2d(*base)
    assert b"taprow" in name2d(*base[:5], 2, 2, *base[7:])            # KW = 2
    assert b"taprow" not in name2d(*base[:5], 1, 1, *base[7:])        # KW = 1: nothing to share
    assert b"taprow" not in name2d(*base[:5], 5, 5, *base[7:])        # KW > 3: stage holds 3 taps
    assert b"taprow" not in name2d(*base[:10], 2, *base[11:])         # dilation 2 in W
    assert b"taprow" not in name2d(*base[:7], 2, 2, *base[9:])        # stride 2: no TMA activations
    h = ctypes.c_void_p()
    d3 = _lib.Conv3dDesc(8, 16, 64, 64, 128, 128, 3, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, _lib.WEIGHTS_ODHWI, 1)
    assert lib.mm4_conv3d_plan_create(ctypes.byref(h), ctypes.byref(d3)) == 0
    assert b"taprow" in lib.mm4_conv_plan_kernel_name(h)
    lib.mm4_conv_plan_destroy(h)
    monkeypatch.setenv("MM4_CONV_TAPREUSE", "0")
    n = name2d(*base)
    assert b"taprow" not in n and b"tma-im2col" in n and b"pair" in n


def test_no_device_means_not_supported():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert _lib.lib().mm4_device_supported() == 0


def test_attention_backward_sizing_and_validation():
    """Host-side contract of the attention backward entry points (no device work): the workspace holds
    the log2-domain LSE and D = rowsum(dO * O) per (batch, query head, row padded to 128), and bad
    arguments are rejected before any launch."""
    lib = _lib.lib()
    h = ctypes.c_void_p()
    a = _lib.AttentionDesc(2, 8, 2, 200, 333, 128, 0.0, _lib.MM4_ATTN_BSHD)
    assert lib.mm4_attention_plan_create(ctypes.byref(h), ctypes.byref(a)) == 0
    ws = lib.mm4_attention_bwd_workspace_size(h)
    assert ws == 2 * 2 * 8 * 256 * 4
    assert lib.mm4_attention_bwd_workspace_size(None) == 0
    fake = 1 << 20  # 16-byte-aligned stand-ins: every check below fails before a pointer is used
    ptrs = [fake] * 9  # Q K V O dO lse dQ dK dV
    assert lib.mm4_attention_bwd(None, *ptrs, fake, ws, None) == _lib.MM4_ERR_INVALID
    for i in range(9):
        bad = list(ptrs)
        bad[i] = None
        assert lib.mm4_attention_bwd(h, *bad, fake, ws, None) == _lib.MM4_ERR_INVALID
    bad = list(ptrs)
    bad[0] = fake + 8
    assert lib.mm4_attention_bwd(h, *bad, fake, ws, None) == _lib.MM4_ERR_INVALID
    assert b"aligned" in lib.mm4_last_error()
    assert lib.mm4_attention_bwd(h, *ptrs, fake, ws - 16, None) == _lib.MM4_ERR_WORKSPACE
    assert lib.mm4_attention_bwd(h, *ptrs, None, ws, None) == _lib.MM4_ERR_WORKSPACE
    assert b"workspace" in lib.mm4_last_error()
    assert lib.mm4_attention_fwd_lse(h, fake, fake, fake, fake, None, None) == _lib.MM4_ERR_INVALID
    lib.mm4_attention_plan_destroy(h)


def test_splitk_group_sizing_and_validation():
    """Host-side checks of the multi-GPU split-K group entry points (no device work)."""
    lib = _lib.lib()
    rc, plan = _gemm(M=512, N=512, K=65536, split_k=32)
    assert rc == 0
    nbytes = ctypes.c_size_t()
    # staging: 2 halves x world slots x [512 rows][512] fp32 (each rank pushes into its slot of the
    # owner's half); flags: ready 128 slices x world, consumed + done 128 each
    for world in (1, 2, 8):
        assert lib.mm4_splitk_group_exchange_bytes(plan, world, ctypes.byref(nbytes)) == 0
        slices = 2 * 2 * 32  # 2 pair tiles x 2 row halves x 32 splits
        assert nbytes.value == 2 * world * 512 * 512 * 4 + slices * world * 8 + 2 * slices * 8
    assert lib.mm4_splitk_group_exchange_bytes(plan, 9, ctypes.byref(nbytes)) == _lib.MM4_ERR_UNSUPPORTED
    assert lib.mm4_splitk_group_exchange_bytes(plan, 0, ctypes.byref(nbytes)) == _lib.MM4_ERR_UNSUPPORTED
    g = ctypes.c_void_p()
    ptrs = (ctypes.c_void_p * 2)(0x100000, 0x200000)
    assert lib.mm4_splitk_group_create(ctypes.byref(g), plan, 2, 2, 0, ptrs, ctypes.c_void_p(0x300000)) == \
        _lib.MM4_ERR_INVALID  # rank out of range
    bad = (ctypes.c_void_p * 2)(0x100000, 0x200010)
    assert lib.mm4_splitk_group_create(ctypes.byref(g), plan, 2, 0, 0, bad, ctypes.c_void_p(0x300000)) == \
        _lib.MM4_ERR_INVALID  # exchange buffers must be 256-byte aligned
    assert b"256-byte" in lib.mm4_last_error()
    lib.mm4_gemm_plan_destroy(plan)
    rc, direct = _gemm(M=512, N=512, K=4096, split_k=1)
    assert lib.mm4_splitk_group_exchange_bytes(direct, 2, ctypes.byref(nbytes)) == _lib.MM4_ERR_UNSUPPORTED
    lib.mm4_gemm_plan_destroy(direct)


def test_comm_and_peer_argument_checks():
    lib = _lib.lib()
    h = ctypes.c_void_p()
    uid = ctypes.create_string_buffer(128)
    assert lib.mm4_comm_init(ctypes.byref(h), 0, 0, uid) == _lib.MM4_ERR_INVALID
    assert lib.mm4_comm_init(ctypes.byref(h), 9, 0, uid) == _lib.MM4_ERR_INVALID
    assert lib.mm4_comm_init(ctypes.byref(h), 2, 2, uid) == _lib.MM4_ERR_INVALID
    assert lib.mm4_comm_init(ctypes.byref(h), 2, 0, None) == _lib.MM4_ERR_INVALID
    p = ctypes.c_void_p()
    assert lib.mm4_peer_alloc(0, ctypes.byref(p), ctypes.byref(_lib.PeerHandle())) == _lib.MM4_ERR_INVALID
    assert lib.mm4_peer_free(None) == 0 and lib.mm4_peer_close(None) == 0
    rc, plan = _gemm(M=512, N=512, K=65536, split_k=32)
    assert lib.mm4_gemm_splitk_run_distributed(plan, None, None, None, None, None, None, 1) == _lib.MM4_ERR_INVALID
    lib.mm4_gemm_plan_destroy(plan)


C_PROBE = r"""
#include "mm4.h"
#include <stdio.h>
int main(void) {
  mm4_gemm_desc d = {512, 512, 65536, 0, 0, 1, 32, 0, 0, 0, 4, 1, 0};
  mm4_gemm_plan* p = NULL;
  if (mm4_gemm_plan_create(&p, &d) != MM4_OK) return 1;
  printf("%s %zu\n", mm4_gemm_plan_kernel_name(p), mm4_gemm_workspace_size(p));
  mm4_gemm_plan_destroy(p);
  mm4_conv3d_desc c = {8, 16, 64, 64, 128, 128, 3, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, MM4_WEIGHTS_ODHWI, 1};
  mm4_conv_plan* cp = NULL;
  if (mm4_conv3d_plan_create(&cp, &c) != MM4_OK) return 2;
  int32_t grid[3];
  if (mm4_conv_plan_tile_grid(cp, grid) != MM4_OK) return 3;
  printf("%s %d %d %d\n", mm4_conv_plan_kernel_name(cp), grid[0], grid[1], grid[2]);
  mm4_conv_plan_destroy(cp);
  return mm4_attention_bwd(NULL, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, NULL) == MM4_ERR_INVALID ? 0 : 4;
}
"""


def test_header_is_plain_c_and_the_library_links_from_c(tmp_path):
    """include/mm4.h is a C header (C99, pedantic) and a C program links libmm4.so and calls it --
    the drop-in boundary as a C or FFI host sees it (host-only calls, no GPU)."""
    import shutil
    import subprocess
    from pathlib import Path
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    root = Path(__file__).resolve().parents[1]
    inc, libdir = root / "include", root / "example_matmul_metal4_b200"
    subprocess.run([cc, "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-fsyntax-only", "-x", "c",
                    str(inc / "mm4.h")], check=True)
    src = tmp_path / "probe.c"
    src.write_text(C_PROBE)
    exe = tmp_path / "probe"
    subprocess.run([cc, "-std=c99", "-Wall", "-Werror", f"-I{inc}", str(src), f"-L{libdir}", "-lmm4",
                    f"-Wl,-rpath,{libdir}", "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, (r.returncode, r.stdout, r.stderr)
    lines = r.stdout.splitlines()
    assert lines[0].startswith("gemm_sm100_pair<") and "splitk" in lines[0]
    assert lines[1].endswith("2112 1 1") and "taprow" in lines[1]


def test_host_buffer_entry_points_validate_before_any_copy():
    """The host-buffer pipelines (mm4_gemm_run_host, mm4_conv_run_host, mm4_attention_fwd_host,
    mm4_attention_bwd_host) reject a null plan, a null buffer and a missing bias or workspace before any
    copy or launch is queued, so these calls need no device."""
    lib = _lib.lib()
    fake = 1 << 20  # stand-in pointers: every call below fails before a pointer is dereferenced
    INVALID, WORKSPACE = _lib.MM4_ERR_INVALID, _lib.MM4_ERR_WORKSPACE

    rc, g = _gemm(M=512, N=256, K=1024, bias=1)
    assert rc == 0
    args = [fake] * 8  # hA hB hbias hC dA dB dbias dC
    assert lib.mm4_gemm_run_host(None, *args, None, 0, 4, None) == INVALID
    for i in range(8):
        bad = list(args)
        bad[i] = None
        assert lib.mm4_gemm_run_host(g, *bad, None, 0, 4, None) == INVALID
    assert b"null" in lib.mm4_last_error()
    lib.mm4_gemm_plan_destroy(g)

    h = ctypes.c_void_p()
    d2 = _lib.Conv2dDesc(3, 9, 9, 16, 32, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, _lib.WEIGHTS_OHWI, 1)
    assert lib.mm4_conv2d_plan_create(ctypes.byref(h), ctypes.byref(d2)) == 0
    args = [fake] * 8  # hx hw hbias hy dx dw dbias dy
    assert lib.mm4_conv_run_host(None, *args, 2, None) == INVALID
    for i in range(8):
        bad = list(args)
        bad[i] = None
        assert lib.mm4_conv_run_host(h, *bad, 2, None) == INVALID
    assert b"bias" in lib.mm4_last_error() or b"null" in lib.mm4_last_error()
    lib.mm4_conv_plan_destroy(h)

    a = _lib.AttentionDesc(2, 8, 2, 200, 333, 128, 0.0, _lib.MM4_ATTN_BSHD)
    assert lib.mm4_attention_plan_create(ctypes.byref(h), ctypes.byref(a)) == 0
    args = [fake] * 8  # hQ hK hV hO dQ dK dV dO
    assert lib.mm4_attention_fwd_host(None, *args, 4, None) == INVALID
    for i in range(8):
        bad = list(args)
        bad[i] = None
        assert lib.mm4_attention_fwd_host(h, *bad, 4, None) == INVALID

    def arr(n, hole=None):
        return (ctypes.c_void_p * n)(*[None if i == hole else fake for i in range(n)])
    ws = lib.mm4_attention_bwd_workspace_size(h)
    assert lib.mm4_attention_bwd_host(None, arr(6), arr(3), arr(6), arr(3), fake, ws, 4, None) == INVALID
    assert lib.mm4_attention_bwd_host(h, None, arr(3), arr(6), arr(3), fake, ws, 4, None) == INVALID
    for i in range(6):
        assert lib.mm4_attention_bwd_host(h, arr(6, i), arr(3), arr(6), arr(3), fake, ws, 4, None) == INVALID
        assert lib.mm4_attention_bwd_host(h, arr(6), arr(3), arr(6, i), arr(3), fake, ws, 4, None) == INVALID
    for i in range(3):
        assert lib.mm4_attention_bwd_host(h, arr(6), arr(3, i), arr(6), arr(3), fake, ws, 4, None) == INVALID
        assert lib.mm4_attention_bwd_host(h, arr(6), arr(3), arr(6), arr(3, i), fake, ws, 4, None) == INVALID
    assert lib.mm4_attention_bwd_host(h, arr(6), arr(3), arr(6), arr(3), None, ws, 4, None) == WORKSPACE
    assert lib.mm4_attention_bwd_host(h, arr(6), arr(3), arr(6), arr(3), fake, ws - 16, 4, None) == WORKSPACE
    assert b"workspace" in lib.mm4_last_error()
    lib.mm4_attention_plan_destroy(h)
